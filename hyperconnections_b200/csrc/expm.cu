// expm.cu — batched exponential of small (n <= 8) float32 matrices.
//
// Layout in registers: a group of G lanes (G = n rounded up to a power of two)
// owns one matrix; lane r of the group holds row r (n floats). A product
// C = A B needs row k of B in every lane, which arrives by __shfl_sync from
// lane k of the same group (n*n shuffles and n*n FMAs per lane). Lanes r >= n
// (padding when n is not a power of two) carry zero rows and are never stored.
//
// Two approximants, both with scaling and squaring:
//  * T18 — the optimised degree-18 Taylor polynomial of Bader, Blanes and
//    Casas, "Computing the Matrix Exponential with an Optimized Taylor
//    Polynomial Approximation", Mathematics 7 (2019) 1174, eq. (15) with the
//    coefficients of that paper, theta_18 = 3.01 for unit roundoff 2^-24. This
//    is the algorithm of the reference's expm_t18
//    (hyperconnections/ops/expm.py:65-106). In "global" mode the scaling
//    exponent is one number for the whole batch, from max_b ||A_b||_1, exactly
//    as the reference computes it (expm.py:81-85); a first kernel writes one
//    partial maximum per CTA into caller-provided scratch and the second reads
//    them all. In "per-matrix" mode every group picks its own exponent.
//  * Pade [7/7] — Higham, "The Scaling and Squaring Method for the Matrix
//    Exponential Revisited", SIAM J. Matrix Anal. Appl. 26 (2005), single
//    precision: theta_7 = 3.925724783138660, per-matrix scaling, the rational
//    approximant r = q^{-1} p solved in registers by Gauss-Jordan elimination
//    with partial pivoting across the lanes of the group. Replaces
//    torch.linalg.matrix_exp at hyperconnections/cghc.py:321.
//
// Backward (both approximants): the gradient of sum(G * f(A)) is the adjoint
// Frechet derivative L_f(A)^*(G), and for a primary matrix function with real
// coefficients L_f(A)^*(G) = L_f(A^T, G). The kernels therefore run the SAME
// evaluation scheme on A^T in forward mode, carrying (X, dX) pairs with
// d(XY) = dX Y + X dY, starting from dA = G / 2^s, and d(r) = q^{-1}(dp - dq r)
// for the rational step (Al-Mohy and Higham, "Computing the Frechet Derivative
// of the Matrix Exponential, with an Application to Condition Number
// Estimation", SIAM J. Matrix Anal. Appl. 30 (2009)). The scaling exponent is
// the forward's (from ||A||_1, not ||A^T||_1).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "generator.cuh"

namespace hc {
namespace {

constexpr int kExpmThreads = 256;

template <int N> struct Group {
  static constexpr int G = N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : 8;
};

// ------------------------------------------------------------ row algebra
// C = A * B (rows in lanes). All 32 lanes must call it (full-mask shuffles).
template <int N, int G>
__device__ __forceinline__ void mm(const float (&a)[N], const float (&b)[N], float (&c)[N]) {
  float out[N];
#pragma unroll
  for (int j = 0; j < N; ++j) out[j] = 0.f;
#pragma unroll
  for (int k = 0; k < N; ++k) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float bkj = __shfl_sync(kFull, b[j], k, G);
      out[j] = fmaf(a[k], bkj, out[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) c[j] = out[j];
}

// (C, dC) = (A B, dA B + A dB)
template <int N, int G>
__device__ __forceinline__ void mm_d(const float (&a)[N], const float (&da)[N], const float (&b)[N],
                                     const float (&db)[N], float (&c)[N], float (&dc)[N]) {
  float o[N], d[N];
#pragma unroll
  for (int j = 0; j < N; ++j) { o[j] = 0.f; d[j] = 0.f; }
#pragma unroll
  for (int k = 0; k < N; ++k) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float bkj = __shfl_sync(kFull, b[j], k, G);
      const float dbkj = __shfl_sync(kFull, db[j], k, G);
      o[j] = fmaf(a[k], bkj, o[j]);
      d[j] = fmaf(da[k], bkj, d[j]);
      d[j] = fmaf(a[k], dbkj, d[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) { c[j] = o[j]; dc[j] = d[j]; }
}

// ||A||_1 = max column sum of |a_ij|; every lane of the group gets it.
template <int N, int G>
__device__ __forceinline__ float norm1_rows(const float (&a)[N]) {
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float s = fabsf(a[j]);
#pragma unroll
    for (int o = 1; o < G; o <<= 1) s += __shfl_xor_sync(kFull, s, o, G);
    m = fmaxf(m, s);
  }
  return m;
}

// ||A||_1 from the rows of A^T: max over rows of A^T of the absolute row sum.
template <int N, int G>
__device__ __forceinline__ float norm1_from_transpose(const float (&at)[N]) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j) s += fabsf(at[j]);
#pragma unroll
  for (int o = 1; o < G; o <<= 1) s = fmaxf(s, __shfl_xor_sync(kFull, s, o, G));
  return s;
}

// Smallest s >= 0 with norm / theta <= 2^s, i.e. ceil(log2(norm/theta))
// clamped at 0, read off the IEEE-754 fields of the fp32 quotient (the
// reference forms the same fp32 quotient, expm.py:82-83).
__device__ __forceinline__ int scaling_exponent(float norm, float theta) {
  if (!(norm > theta)) return 0;  // also NaN -> 0; NaNs propagate through the math
  const float ratio = norm / theta;
  const uint32_t bits = __float_as_uint(ratio);
  const int e = static_cast<int>((bits >> 23) & 0xffu) - 127;
  const uint32_t mant = bits & 0x7fffffu;
  int s = e + (mant != 0u ? 1 : 0);
  if (s > 126) s = 126;
  return s < 0 ? 0 : s;
}

__device__ __forceinline__ float pow2_neg(int s) {  // exact 2^-s for 0 <= s <= 126
  return __uint_as_float(static_cast<uint32_t>(127 - s) << 23);
}

// ------------------------------------------------------------ T18 scheme
// Coefficients of eq. (15) of Bader, Blanes and Casas (2019); a01, b01, b04
// and b14 are zero.
constexpr float kA11 = -0.10036558103014462f, kA21 = -0.008029246482411570f,
                kA31 = -0.000892138498045730f;
constexpr float kB11 = 0.39784974949645076f, kB21 = 1.36783778460411719f,
                kB31 = 0.49828962252538268f, kB61 = -0.00063789819459247233f;
constexpr float kB02 = -10.96763960529620626f, kB12 = 1.68015813878906197f,
                kB22 = 0.05717798464788655f, kB32 = -0.00698210122488052f,
                kB62 = 0.00003349750170860705f;
constexpr float kB03 = -0.09043168323908106f, kB13 = -0.06764045190713819f,
                kB23 = 0.06759613017740597f, kB33 = 0.02955525704293155f,
                kB63 = -0.00001391802575160607f;
constexpr float kB24 = -0.09233646193671186f, kB34 = -0.01693649390020817f,
                kB64 = -0.00001400867981820361f;
constexpr float kTheta18 = 3.01f;

// One row of c0*I + c1*X1 + c2*X2 + c3*X3 + c6*X6 (the I term sits on the
// diagonal entry r of this lane's row).
template <int N>
__device__ __forceinline__ void combo(float (&o)[N], int r, float c0, float c1, const float (&x1)[N],
                                      float c2, const float (&x2)[N], float c3, const float (&x3)[N],
                                      float c6, const float (&x6)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float s = c1 * x1[j];
    s = fmaf(c2, x2[j], s);
    s = fmaf(c3, x3[j], s);
    s = fmaf(c6, x6[j], s);
    o[j] = s + (j == r ? c0 : 0.f);
  }
}

// Derivative rows of the same combination (no identity term).
template <int N>
__device__ __forceinline__ void dcombo(float (&o)[N], float c1, const float (&x1)[N], float c2,
                                       const float (&x2)[N], float c3, const float (&x3)[N], float c6,
                                       const float (&x6)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float s = c1 * x1[j];
    s = fmaf(c2, x2[j], s);
    s = fmaf(c3, x3[j], s);
    o[j] = fmaf(c6, x6[j], s);
  }
}

template <int N, int G>
__device__ __forceinline__ void t18_eval(const float (&a)[N], int r, float (&t)[N]) {
  float a2[N], a3[N], a6[N];
  mm<N, G>(a, a, a2);
  mm<N, G>(a2, a, a3);
  mm<N, G>(a3, a3, a6);
  const float z[N] = {};
  float b1[N], b4[N], b5[N], a9[N];
  combo<N>(b1, r, 0.f, kA11, a, kA21, a2, kA31, a3, 0.f, z);
  combo<N>(b5, r, 0.f, 0.f, a, kB24, a2, kB34, a3, kB64, a6);
  combo<N>(b4, r, kB03, kB13, a, kB23, a2, kB33, a3, kB63, a6);
  mm<N, G>(b1, b5, a9);
#pragma unroll
  for (int j = 0; j < N; ++j) a9[j] += b4[j];
  float b2[N], b3[N];
  combo<N>(b2, r, 0.f, kB11, a, kB21, a2, kB31, a3, kB61, a6);
  combo<N>(b3, r, kB02, kB12, a, kB22, a2, kB32, a3, kB62, a6);
#pragma unroll
  for (int j = 0; j < N; ++j) b3[j] += a9[j];
  float p[N];
  mm<N, G>(b3, a9, p);
#pragma unroll
  for (int j = 0; j < N; ++j) t[j] = b2[j] + p[j];
}

template <int N, int G>
__device__ __forceinline__ void t18_eval_d(const float (&a)[N], const float (&da)[N], int r,
                                           float (&t)[N], float (&dt)[N]) {
  float a2[N], a3[N], a6[N], d2[N], d3[N], d6[N];
  mm_d<N, G>(a, da, a, da, a2, d2);
  mm_d<N, G>(a2, d2, a, da, a3, d3);
  mm_d<N, G>(a3, d3, a3, d3, a6, d6);
  const float z[N] = {};
  float b1[N], b4[N], b5[N], db1[N], db4[N], db5[N];
  combo<N>(b1, r, 0.f, kA11, a, kA21, a2, kA31, a3, 0.f, z);
  dcombo<N>(db1, kA11, da, kA21, d2, kA31, d3, 0.f, z);
  combo<N>(b5, r, 0.f, 0.f, a, kB24, a2, kB34, a3, kB64, a6);
  dcombo<N>(db5, 0.f, da, kB24, d2, kB34, d3, kB64, d6);
  combo<N>(b4, r, kB03, kB13, a, kB23, a2, kB33, a3, kB63, a6);
  dcombo<N>(db4, kB13, da, kB23, d2, kB33, d3, kB63, d6);
  float a9[N], d9[N];
  mm_d<N, G>(b1, db1, b5, db5, a9, d9);
#pragma unroll
  for (int j = 0; j < N; ++j) { a9[j] += b4[j]; d9[j] += db4[j]; }
  float b2[N], b3[N], db2[N], db3[N];
  combo<N>(b2, r, 0.f, kB11, a, kB21, a2, kB31, a3, kB61, a6);
  dcombo<N>(db2, kB11, da, kB21, d2, kB31, d3, kB61, d6);
  combo<N>(b3, r, kB02, kB12, a, kB22, a2, kB32, a3, kB62, a6);
  dcombo<N>(db3, kB12, da, kB22, d2, kB32, d3, kB62, d6);
#pragma unroll
  for (int j = 0; j < N; ++j) { b3[j] += a9[j]; db3[j] += d9[j]; }
  float p[N], dp[N];
  mm_d<N, G>(b3, db3, a9, d9, p, dp);
#pragma unroll
  for (int j = 0; j < N; ++j) { t[j] = b2[j] + p[j]; dt[j] = db2[j] + dp[j]; }
}

// ------------------------------------------------------------ Pade [7/7]
// p(x) = sum_k c_k x^k with c_k = (14-k)! 7! / (14! k! (7-k)!), scaled by 14!/7!
constexpr float kP0 = 17297280.f, kP1 = 8648640.f, kP2 = 1995840.f, kP3 = 277200.f,
                kP4 = 25200.f, kP5 = 1512.f, kP6 = 56.f, kP7 = 1.f;
constexpr float kTheta7 = 3.925724783138660f;

// Gauss-Jordan on [Q | B_0 | ... | B_{K-1}] (rows in lanes, partial
// pivoting); on return lane r holds row r of Q^{-1} B_k for every k.
template <int N, int G, int K>
__device__ __forceinline__ void gj_solve(float (&q)[N], float (&b)[K][N], int lane_in_group) {
  int rowid = lane_in_group;  // logical row this lane currently holds
#pragma unroll
  for (int k = 0; k < N; ++k) {
    // pivot: largest |q[k]| among logical rows >= k (ties -> lower lane)
    float best = (rowid >= k && lane_in_group < N) ? fabsf(q[k]) : -1.f;
    int bl = lane_in_group;
#pragma unroll
    for (int o = 1; o < G; o <<= 1) {
      const float ob = __shfl_xor_sync(kFull, best, o, G);
      const int ol = __shfl_xor_sync(kFull, bl, o, G);
      if (ob > best || (ob == best && ol < bl)) { best = ob; bl = ol; }
    }
    // broadcast the pivot row
    float pr[N], pb[K][N];
#pragma unroll
    for (int j = 0; j < N; ++j) pr[j] = __shfl_sync(kFull, q[j], bl, G);
#pragma unroll
    for (int kk = 0; kk < K; ++kk)
#pragma unroll
      for (int j = 0; j < N; ++j) pb[kk][j] = __shfl_sync(kFull, b[kk][j], bl, G);
    // swap logical ids of the pivot lane and the lane that held row k
    const int pivot_rowid = __shfl_sync(kFull, rowid, bl, G);
    if (lane_in_group == bl) {
      rowid = k;
    } else if (rowid == k) {
      rowid = pivot_rowid;
    }
    // eliminate column k from every other row
    if (lane_in_group != bl) {
      const float f = q[k] / pr[k];
#pragma unroll
      for (int j = 0; j < N; ++j) q[j] = fmaf(-f, pr[j], q[j]);
#pragma unroll
      for (int kk = 0; kk < K; ++kk)
#pragma unroll
        for (int j = 0; j < N; ++j) b[kk][j] = fmaf(-f, pb[kk][j], b[kk][j]);
    }
  }
  // divide by the diagonal: the lane holding logical row rid has q[rid] != 0
  float diag = 1.f;
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (j == rowid) diag = q[j];
  if (lane_in_group < N) {
    const float inv = 1.f / diag;
#pragma unroll
    for (int kk = 0; kk < K; ++kk)
#pragma unroll
      for (int j = 0; j < N; ++j) b[kk][j] *= inv;
  }
  // move logical row r into lane r
  int src = lane_in_group;
#pragma unroll
  for (int l = 0; l < G; ++l) {
    const int rid = __shfl_sync(kFull, rowid, l, G);
    if (rid == lane_in_group) src = l;
  }
#pragma unroll
  for (int kk = 0; kk < K; ++kk)
#pragma unroll
    for (int j = 0; j < N; ++j) b[kk][j] = __shfl_sync(kFull, b[kk][j], src, G);
}

template <int N, int G>
__device__ __forceinline__ void pade7_eval(const float (&a)[N], int r, float (&out)[N]) {
  float a2[N], a4[N], a6[N];
  mm<N, G>(a, a, a2);
  mm<N, G>(a2, a2, a4);
  mm<N, G>(a4, a2, a6);
  float w[N], v[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float s = kP7 * a6[j];
    s = fmaf(kP5, a4[j], s);
    s = fmaf(kP3, a2[j], s);
    w[j] = s + (j == r ? kP1 : 0.f);
    float t = kP6 * a6[j];
    t = fmaf(kP4, a4[j], t);
    t = fmaf(kP2, a2[j], t);
    v[j] = t + (j == r ? kP0 : 0.f);
  }
  float u[N];
  mm<N, G>(a, w, u);
  float q[N], b[1][N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    b[0][j] = v[j] + u[j];
    q[j] = v[j] - u[j];
  }
  gj_solve<N, G, 1>(q, b, r);
#pragma unroll
  for (int j = 0; j < N; ++j) out[j] = b[0][j];
}

template <int N, int G>
__device__ __forceinline__ void pade7_eval_d(const float (&a)[N], const float (&da)[N], int r,
                                             float (&out)[N], float (&dout)[N]) {
  float a2[N], a4[N], a6[N], d2[N], d4[N], d6[N];
  mm_d<N, G>(a, da, a, da, a2, d2);
  mm_d<N, G>(a2, d2, a2, d2, a4, d4);
  mm_d<N, G>(a4, d4, a2, d2, a6, d6);
  float w[N], v[N], dw[N], dv[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float s = kP7 * a6[j];
    s = fmaf(kP5, a4[j], s);
    s = fmaf(kP3, a2[j], s);
    w[j] = s + (j == r ? kP1 : 0.f);
    float ds = kP7 * d6[j];
    ds = fmaf(kP5, d4[j], ds);
    dw[j] = fmaf(kP3, d2[j], ds);
    float t = kP6 * a6[j];
    t = fmaf(kP4, a4[j], t);
    t = fmaf(kP2, a2[j], t);
    v[j] = t + (j == r ? kP0 : 0.f);
    float dt = kP6 * d6[j];
    dt = fmaf(kP4, d4[j], dt);
    dv[j] = fmaf(kP2, d2[j], dt);
  }
  float u[N], du[N];
  mm_d<N, G>(a, da, w, dw, u, du);
  // solve Q [R | X1 | X2] = [P | dP | dQ]
  float q[N], b[3][N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    b[0][j] = v[j] + u[j];
    q[j] = v[j] - u[j];
    b[1][j] = dv[j] + du[j];
    b[2][j] = dv[j] - du[j];
  }
  gj_solve<N, G, 3>(q, b, r);
  // dR = X1 - X2 R
  float x2r[N];
  mm<N, G>(b[2], b[0], x2r);
#pragma unroll
  for (int j = 0; j < N; ++j) {
    out[j] = b[0][j];
    dout[j] = b[1][j] - x2r[j];
  }
}

// ------------------------------------------------------------ kernels
template <int N>
__device__ __forceinline__ void load_row(const float* __restrict__ base, int64_t m, int64_t batch, int r,
                                         float (&row)[N]) {
  const bool ok = m < batch && r < N;
  const float* p = base + m * (N * N) + r * N;
#pragma unroll
  for (int j = 0; j < N; ++j) row[j] = ok ? __ldg(p + j) : 0.f;
}

// Column r of the matrix = row r of its transpose.
template <int N>
__device__ __forceinline__ void load_col(const float* __restrict__ base, int64_t m, int64_t batch, int r,
                                         float (&row)[N]) {
  const bool ok = m < batch && r < N;
  const float* p = base + m * (N * N) + r;
#pragma unroll
  for (int j = 0; j < N; ++j) row[j] = ok ? __ldg(p + j * N) : 0.f;
}

template <int N>
__device__ __forceinline__ void store_row(float* __restrict__ base, int64_t m, int64_t batch, int r,
                                          const float (&row)[N]) {
  if (m >= batch || r >= N) return;
  float* p = base + m * (N * N) + r * N;
#pragma unroll
  for (int j = 0; j < N; ++j) p[j] = row[j];
}

// Squarings: X <- X^2 while i < s. s may differ between groups of one warp,
// so the loop runs to the warp maximum and every lane keeps shuffling.
template <int N, int G>
__device__ __forceinline__ void square_s(float (&x)[N], int s) {
  const int smax = __reduce_max_sync(kFull, s);
  for (int i = 0; i < smax; ++i) {
    float y[N];
    mm<N, G>(x, x, y);
    if (i < s) {
#pragma unroll
      for (int j = 0; j < N; ++j) x[j] = y[j];
    }
  }
}

template <int N, int G>
__device__ __forceinline__ void square_s_d(float (&x)[N], float (&dx)[N], int s) {
  const int smax = __reduce_max_sync(kFull, s);
  for (int i = 0; i < smax; ++i) {
    float y[N], dy[N];
    mm_d<N, G>(x, dx, x, dx, y, dy);
    if (i < s) {
#pragma unroll
      for (int j = 0; j < N; ++j) { x[j] = y[j]; dx[j] = dy[j]; }
    }
  }
}

// Partial maxima of ||A_b||_1, one per CTA (grid-stride over matrices).
template <int N>
__global__ void __launch_bounds__(kExpmThreads) expm_norm_partial_kernel(const float* __restrict__ A,
                                                                         int64_t batch,
                                                                         float* __restrict__ partial) {
  constexpr int G = Group<N>::G;
  __shared__ float wmax[kExpmThreads / 32];
  const int lane = threadIdx.x & 31;
  const int r = lane & (G - 1);
  const int64_t per_cta = kExpmThreads / G;
  float m = 0.f;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * per_cta; base < batch;
       base += static_cast<int64_t>(gridDim.x) * per_cta) {
    const int64_t mat = base + threadIdx.x / G;
    float a[N];
    load_row<N>(A, mat, batch, r, a);
    m = fmaxf(m, norm1_rows<N, G>(a));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
  if (lane == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.f;
    for (int w = 0; w < kExpmThreads / 32; ++w) b = fmaxf(b, wmax[w]);
    partial[blockIdx.x] = b;
  }
}

// Global scaling exponent from the partial maxima (every CTA reduces them).
__device__ __forceinline__ int global_exponent(const float* __restrict__ partial, int nparts, float theta) {
  __shared__ float smax[kExpmThreads / 32];
  float m = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) m = fmaxf(m, __ldg(partial + i));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
  if ((threadIdx.x & 31) == 0) smax[threadIdx.x >> 5] = m;
  __syncthreads();
  float b = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) b = fmaxf(b, smax[w]);
  return scaling_exponent(b, theta);
}

template <int N>
__global__ void __launch_bounds__(kExpmThreads) expm_t18_fwd_kernel(const float* __restrict__ A,
                                                                    float* __restrict__ E, int64_t batch,
                                                                    const float* __restrict__ partial,
                                                                    int nparts) {
  constexpr int G = Group<N>::G;
  const int s_glob = partial ? global_exponent(partial, nparts, kTheta18) : 0;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t mat = gt / G;
  const int r = static_cast<int>(gt & (G - 1));
  float a[N];
  load_row<N>(A, mat, batch, r, a);
  const int s = partial ? s_glob : scaling_exponent(norm1_rows<N, G>(a), kTheta18);
  const float sc = pow2_neg(s);
#pragma unroll
  for (int j = 0; j < N; ++j) a[j] *= sc;
  float t[N];
  t18_eval<N, G>(a, r, t);
  square_s<N, G>(t, s);
  store_row<N>(E, mat, batch, r, t);
}

template <int N>
__global__ void __launch_bounds__(kExpmThreads) expm_t18_bwd_kernel(const float* __restrict__ A,
                                                                    const float* __restrict__ Gr,
                                                                    float* __restrict__ dA, int64_t batch,
                                                                    const float* __restrict__ partial,
                                                                    int nparts) {
  constexpr int G = Group<N>::G;
  const int s_glob = partial ? global_exponent(partial, nparts, kTheta18) : 0;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t mat = gt / G;
  const int r = static_cast<int>(gt & (G - 1));
  float at[N], e[N];
  load_col<N>(A, mat, batch, r, at);  // row r of A^T
  load_row<N>(Gr, mat, batch, r, e);  // direction G
  const int s = partial ? s_glob : scaling_exponent(norm1_from_transpose<N, G>(at), kTheta18);
  const float sc = pow2_neg(s);
#pragma unroll
  for (int j = 0; j < N; ++j) { at[j] *= sc; e[j] *= sc; }
  float t[N], dt[N];
  t18_eval_d<N, G>(at, e, r, t, dt);
  square_s_d<N, G>(t, dt, s);
  store_row<N>(dA, mat, batch, r, dt);
}

// ------------------------------------------------ one thread per matrix (n <= 4)
// For n <= 4 a whole matrix (at most 16 floats) fits one thread's registers,
// and a product is n^3 FMAs with no shuffle at all. These helpers perform the
// operations of the row-per-lane scheme above element for element, in the
// same order (products accumulate over k ascending from 0; the column sums of
// ||A||_1 add rows pairwise as the xor-shuffle tree does; the identity term
// is added as `s + c0` or `s + 0`), so the forward below returns bitwise the
// results of expm_t18_fwd_kernel.
template <int N>
__device__ __forceinline__ void tm_mm(const float (&a)[N][N], const float (&b)[N][N], float (&c)[N][N]) {
  float o[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) o[i][j] = 0.f;
#pragma unroll
  for (int k = 0; k < N; ++k)
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) o[i][j] = fmaf(a[i][k], b[k][j], o[i][j]);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) c[i][j] = o[i][j];
}

template <int N>
__device__ __forceinline__ void tm_combo(float (&o)[N][N], float c0, float c1, const float (&x1)[N][N], float c2,
                                         const float (&x2)[N][N], float c3, const float (&x3)[N][N], float c6,
                                         const float (&x6)[N][N]) {
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float s = c1 * x1[i][j];
      s = fmaf(c2, x2[i][j], s);
      s = fmaf(c3, x3[i][j], s);
      s = fmaf(c6, x6[i][j], s);
      o[i][j] = s + (j == i ? c0 : 0.f);
    }
}

// T18 from the powers a, a2 = a a, a3 = a2 a, a6 = a3 a3 (the combinations
// and the two remaining products).
template <int N>
__device__ __forceinline__ void tm_t18_tail(const float (&a)[N][N], const float (&a2)[N][N],
                                            const float (&a3)[N][N], const float (&a6)[N][N], float (&t)[N][N]) {
  const float z[N][N] = {};
  float b1[N][N], b4[N][N], b5[N][N], a9[N][N];
  tm_combo<N>(b1, 0.f, kA11, a, kA21, a2, kA31, a3, 0.f, z);
  tm_combo<N>(b5, 0.f, 0.f, a, kB24, a2, kB34, a3, kB64, a6);
  tm_combo<N>(b4, kB03, kB13, a, kB23, a2, kB33, a3, kB63, a6);
  tm_mm<N>(b1, b5, a9);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) a9[i][j] += b4[i][j];
  float b2[N][N], b3[N][N];
  tm_combo<N>(b2, 0.f, kB11, a, kB21, a2, kB31, a3, kB61, a6);
  tm_combo<N>(b3, kB02, kB12, a, kB22, a2, kB32, a3, kB62, a6);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) b3[i][j] += a9[i][j];
  float p[N][N];
  tm_mm<N>(b3, a9, p);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) t[i][j] = b2[i][j] + p[i][j];
}

template <int N>
__device__ __forceinline__ void tm_powers(const float (&a)[N][N], float (&a2)[N][N], float (&a3)[N][N],
                                          float (&a6)[N][N]) {
  tm_mm<N>(a, a, a2);
  tm_mm<N>(a2, a, a3);
  tm_mm<N>(a3, a3, a6);
}

template <int N>
__device__ __forceinline__ void tm_t18(const float (&a)[N][N], float (&t)[N][N]) {
  float a2[N][N], a3[N][N], a6[N][N];
  tm_powers<N>(a, a2, a3, a6);
  tm_t18_tail<N>(a, a2, a3, a6, t);
}

template <int N>
__device__ __forceinline__ void tm_scale(float (&x)[N][N], float c) {
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) x[i][j] *= c;
}

// (C, dC) = (A B, dA B + A dB), the per-element order of mm_d.
template <int N>
__device__ __forceinline__ void tm_mm_d(const float (&a)[N][N], const float (&da)[N][N], const float (&b)[N][N],
                                        const float (&db)[N][N], float (&c)[N][N], float (&dc)[N][N]) {
  float o[N][N], d[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      o[i][j] = 0.f;
      d[i][j] = 0.f;
    }
#pragma unroll
  for (int k = 0; k < N; ++k)
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) {
        o[i][j] = fmaf(a[i][k], b[k][j], o[i][j]);
        d[i][j] = fmaf(da[i][k], b[k][j], d[i][j]);
        d[i][j] = fmaf(a[i][k], db[k][j], d[i][j]);
      }
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      c[i][j] = o[i][j];
      dc[i][j] = d[i][j];
    }
}

template <int N>
__device__ __forceinline__ void tm_dcombo(float (&o)[N][N], float c1, const float (&x1)[N][N], float c2,
                                          const float (&x2)[N][N], float c3, const float (&x3)[N][N], float c6,
                                          const float (&x6)[N][N]) {
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float s = c1 * x1[i][j];
      s = fmaf(c2, x2[i][j], s);
      s = fmaf(c3, x3[i][j], s);
      o[i][j] = fmaf(c6, x6[i][j], s);
    }
}

// T18 and its forward-mode derivative in direction da, the steps of
// t18_eval_d.
template <int N>
__device__ __forceinline__ void tm_t18_d(const float (&a)[N][N], const float (&da)[N][N], float (&t)[N][N],
                                         float (&dt)[N][N]) {
  float a2[N][N], a3[N][N], a6[N][N], d2[N][N], d3[N][N], d6[N][N];
  tm_mm_d<N>(a, da, a, da, a2, d2);
  tm_mm_d<N>(a2, d2, a, da, a3, d3);
  tm_mm_d<N>(a3, d3, a3, d3, a6, d6);
  const float z[N][N] = {};
  float b1[N][N], b5[N][N], db1[N][N], db5[N][N];
  tm_combo<N>(b1, 0.f, kA11, a, kA21, a2, kA31, a3, 0.f, z);
  tm_dcombo<N>(db1, kA11, da, kA21, d2, kA31, d3, 0.f, z);
  tm_combo<N>(b5, 0.f, 0.f, a, kB24, a2, kB34, a3, kB64, a6);
  tm_dcombo<N>(db5, 0.f, da, kB24, d2, kB34, d3, kB64, d6);
  float a9[N][N], d9[N][N];
  tm_mm_d<N>(b1, db1, b5, db5, a9, d9);
  {
    float b4[N][N], db4[N][N];
    tm_combo<N>(b4, kB03, kB13, a, kB23, a2, kB33, a3, kB63, a6);
    tm_dcombo<N>(db4, kB13, da, kB23, d2, kB33, d3, kB63, d6);
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) {
        a9[i][j] += b4[i][j];
        d9[i][j] += db4[i][j];
      }
  }
  float b2[N][N], b3[N][N], db2[N][N], db3[N][N];
  tm_combo<N>(b2, 0.f, kB11, a, kB21, a2, kB31, a3, kB61, a6);
  tm_dcombo<N>(db2, kB11, da, kB21, d2, kB31, d3, kB61, d6);
  tm_combo<N>(b3, kB02, kB12, a, kB22, a2, kB32, a3, kB62, a6);
  tm_dcombo<N>(db3, kB12, da, kB22, d2, kB32, d3, kB62, d6);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      b3[i][j] += a9[i][j];
      db3[i][j] += d9[i][j];
    }
  float p[N][N], dp[N][N];
  tm_mm_d<N>(b3, db3, a9, d9, p, dp);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      t[i][j] = b2[i][j] + p[i][j];
      dt[i][j] = db2[i][j] + dp[i][j];
    }
}

// ||A||_1: column sums of |a_ij| over the rows added pairwise (row 0 + row 1,
// row 2 + row 3, then the two), the order of the xor-shuffle tree of
// norm1_rows; a missing fourth row of n = 3 adds an exact zero there too.
template <int N>
__device__ __forceinline__ float tm_norm1(const float (&a)[N][N]) {
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float s;
    if constexpr (N == 1) {
      s = fabsf(a[0][j]);
    } else if constexpr (N == 2) {
      s = fabsf(a[0][j]) + fabsf(a[1][j]);
    } else if constexpr (N == 3) {
      s = (fabsf(a[0][j]) + fabsf(a[1][j])) + (fabsf(a[2][j]) + 0.f);
    } else {
      s = (fabsf(a[0][j]) + fabsf(a[1][j])) + (fabsf(a[2][j]) + fabsf(a[3][j]));
    }
    m = fmaxf(m, s);
  }
  return m;
}

template <int N>
__device__ __forceinline__ void tm_load(const float* __restrict__ base, int64_t m, bool vec, float (&a)[N][N]) {
  const float* p = base + m * (N * N);
  if constexpr ((N * N) % 4 == 0) {
    if (vec) {
#pragma unroll
      for (int q = 0; q < N * N / 4; ++q) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p) + q);
        const float w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) a[(4 * q + e) / N][(4 * q + e) % N] = w[e];
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) a[i][j] = __ldg(p + i * N + j);
}

template <int N>
__device__ __forceinline__ void tm_store(float* __restrict__ base, int64_t m, bool vec, const float (&a)[N][N]) {
  float* p = base + m * (N * N);
  if constexpr ((N * N) % 4 == 0) {
    if (vec) {
#pragma unroll
      for (int q = 0; q < N * N / 4; ++q) {
        float4 v;
        v.x = a[(4 * q) / N][(4 * q) % N];
        v.y = a[(4 * q + 1) / N][(4 * q + 1) % N];
        v.z = a[(4 * q + 2) / N][(4 * q + 2) % N];
        v.w = a[(4 * q + 3) / N][(4 * q + 3) % N];
        reinterpret_cast<float4*>(p)[q] = v;
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) p[i * N + j] = a[i][j];
}

// Largest batch exponent for which the first matrix's powers formed before
// the grid barrier are used (||A||_1 <= 3.01 * 2^10: A^6 stays far from
// overflow, and A^6 2^-60 from the subnormal range for entries of interest).
constexpr int kSpecMaxS = 10;

// Count of bounded waits that gave up (read and cleared by hc_wait_timeouts()).
__device__ unsigned int g_expm_wait_timeouts;

// Grid-wide barrier of a cooperative launch (every CTA is resident, so every
// arrival comes), split in two so that a CTA can work between arriving and
// waiting. `count` is zeroed by the host before the launch. Bounded (`limit`
// polls of ~64 ns; kWaitPolls is a quarter of a second): a CTA that gives up
// counts it in g_expm_wait_timeouts and in the library's status word (the
// next entry point call returns HC_ERR_TIMEOUT) and goes on with the partial
// maxima it has seen, so that batch's exponent may be too small.
__device__ __forceinline__ void grid_arrive(unsigned int* count) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // this CTA's partial maximum is visible to every CTA
    atomicAdd(count, 1u);
  }
}

__device__ __forceinline__ void grid_wait(unsigned int* count, uint32_t limit, unsigned int* status) {
  if (threadIdx.x == 0) {
    bool ok = false;
    for (uint32_t i = 0; i < limit; ++i) {
      unsigned int seen;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(count) : "memory");
      if (seen >= gridDim.x) {
        ok = true;
        break;
      }
      __nanosleep(64);
    }
    if (!ok) report_timeout(&g_expm_wait_timeouts, status);
  }
  __syncthreads();
}

// T18 forward, one thread per matrix, grid-stride over the batch, with the
// scaling exponent per matrix (partial == nullptr) or, for the reference's
// global scaling, from the partial maxima of ||A||_1 of a previous norm pass.
template <int N>
__global__ void __launch_bounds__(kExpmThreads) expm_t18_tm_fwd_kernel(const float* __restrict__ A,
                                                                       float* __restrict__ E, int64_t batch,
                                                                       const float* __restrict__ partial,
                                                                       int nparts, int vec) {
  const int s_glob = partial ? global_exponent(partial, nparts, kTheta18) : 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t mat = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; mat < batch; mat += stride) {
    float a[N][N];
    tm_load<N>(A, mat, vec != 0, a);
    const int s = partial ? s_glob : scaling_exponent(tm_norm1<N>(a), kTheta18);
    tm_scale<N>(a, pow2_neg(s));
    float t[N][N];
    tm_t18<N>(a, t);
    for (int i = 0; i < s; ++i) tm_mm<N>(t, t, t);
    tm_store<N>(E, mat, vec != 0, t);
  }
}

// T18 forward with the reference's global scaling in ONE launch, one thread
// per matrix (batch <= gridDim.x * blockDim.x): every CTA writes the maximum
// ||A||_1 of its matrices to partial[blockIdx.x] and arrives at a grid barrier
// (the launch is cooperative); while the barrier completes each thread forms
// the powers A^2, A^3, A^6 of its matrix unscaled; every CTA then reduces all
// partials to the batch's exponent s. Scaling by 2^-s commutes with every
// rounded product and sum of those powers (power-of-two factors; for
// s <= kSpecMaxS nothing overflows or becomes subnormal), so scaling them by
// 2^-2s, 2^-3s, 2^-6s gives bit for bit the powers of A / 2^s; for larger s
// the powers are formed again from A / 2^s.
template <int N>
__global__ void __launch_bounds__(kExpmThreads) expm_t18_tm_coop_kernel(const float* __restrict__ A,
                                                                        float* __restrict__ E, int64_t batch,
                                                                        float* __restrict__ partial,
                                                                        unsigned int* __restrict__ arrive,
                                                                        int vec, uint32_t wait_limit,
                                                                        unsigned int* status) {
  __shared__ float wmax[kExpmThreads / 32];
  const int64_t mat = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool live = mat < batch;
  float a[N][N];
  tm_load<N>(A, live ? mat : 0, vec != 0, a);
  float m = live ? tm_norm1<N>(a) : 0.f;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.f;
    for (int w = 0; w < kExpmThreads / 32; ++w) b = fmaxf(b, wmax[w]);
    partial[blockIdx.x] = b;
  }
  grid_arrive(arrive);
  float p2[N][N], p3[N][N], p6[N][N];
  tm_powers<N>(a, p2, p3, p6);
  grid_wait(arrive, wait_limit, status);
  float g = 0.f;
  for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += blockDim.x) g = fmaxf(g, __ldcg(partial + i));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) g = fmaxf(g, __shfl_xor_sync(kFull, g, o));
  __syncthreads();  // wmax is reused
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = g;
  __syncthreads();
  float b = 0.f;
  for (int w = 0; w < kExpmThreads / 32; ++w) b = fmaxf(b, wmax[w]);
  const int s = scaling_exponent(b, kTheta18);
  if (!live) return;
  tm_scale<N>(a, pow2_neg(s));
  if (s <= kSpecMaxS) {
    tm_scale<N>(p2, pow2_neg(2 * s));
    tm_scale<N>(p3, pow2_neg(3 * s));
    tm_scale<N>(p6, pow2_neg(6 * s));
  } else {
    tm_powers<N>(a, p2, p3, p6);
  }
  float t[N][N];
  tm_t18_tail<N>(a, p2, p3, p6, t);
  for (int i = 0; i < s; ++i) tm_mm<N>(t, t, t);
  tm_store<N>(E, mat, vec != 0, t);
}

// T18 backward, one thread per matrix: the adjoint Frechet derivative
// L(A^T, G) in forward mode, bitwise the result of expm_t18_bwd_kernel. The
// (X, dX) pairs need ~230 live floats, so CTAs are small and each thread
// stays close to the 255-register limit.
constexpr int kExpmTmBwdThreads = 128;

template <int N>
__global__ void __launch_bounds__(kExpmTmBwdThreads) expm_t18_tm_bwd_kernel(const float* __restrict__ A,
                                                                            const float* __restrict__ Gr,
                                                                            float* __restrict__ dA, int64_t batch,
                                                                            const float* __restrict__ partial,
                                                                            int nparts, int vec) {
  // The matrix loads go out first, so that their latency overlaps the
  // reduction of the partial maxima (which ends in a CTA barrier).
  const int64_t mat = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool live = mat < batch;
  float at[N][N], e[N][N];
  {
    float a[N][N];
    tm_load<N>(A, live ? mat : 0, vec != 0, a);
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) at[i][j] = a[j][i];
  }
  tm_load<N>(Gr, live ? mat : 0, vec != 0, e);
  const int s_glob = partial ? global_exponent(partial, nparts, kTheta18) : 0;
  if (!live) return;
  int s = s_glob;
  if (!partial) {  // ||A||_1 as the max row sum of A^T, summed as norm1_from_transpose does
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float r = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) r += fabsf(at[i][j]);
      m = fmaxf(m, r);
    }
    s = scaling_exponent(m, kTheta18);
  }
  const float sc = pow2_neg(s);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      at[i][j] *= sc;
      e[i][j] *= sc;
    }
  float t[N][N], dt[N][N];
  tm_t18_d<N>(at, e, t, dt);
  for (int i = 0; i < s; ++i) tm_mm_d<N>(t, dt, t, dt, t, dt);
  tm_store<N>(dA, mat, vec != 0, dt);
}

template <int N>
__global__ void __launch_bounds__(kExpmThreads) expm_pade_fwd_kernel(const float* __restrict__ A,
                                                                     float* __restrict__ E, int64_t batch) {
  constexpr int G = Group<N>::G;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t mat = gt / G;
  const int r = static_cast<int>(gt & (G - 1));
  float a[N];
  load_row<N>(A, mat, batch, r, a);
  const int s = scaling_exponent(norm1_rows<N, G>(a), kTheta7);
  const float sc = pow2_neg(s);
#pragma unroll
  for (int j = 0; j < N; ++j) a[j] *= sc;
  float t[N];
  pade7_eval<N, G>(a, r, t);
  square_s<N, G>(t, s);
  store_row<N>(E, mat, batch, r, t);
}

template <int N>
__global__ void __launch_bounds__(kExpmThreads) expm_pade_bwd_kernel(const float* __restrict__ A,
                                                                     const float* __restrict__ Gr,
                                                                     float* __restrict__ dA, int64_t batch) {
  constexpr int G = Group<N>::G;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t mat = gt / G;
  const int r = static_cast<int>(gt & (G - 1));
  float at[N], e[N];
  load_col<N>(A, mat, batch, r, at);
  load_row<N>(Gr, mat, batch, r, e);
  const int s = scaling_exponent(norm1_from_transpose<N, G>(at), kTheta7);
  const float sc = pow2_neg(s);
#pragma unroll
  for (int j = 0; j < N; ++j) { at[j] *= sc; e[j] *= sc; }
  float t[N], dt[N];
  pade7_eval_d<N, G>(at, e, r, t, dt);
  square_s_d<N, G>(t, dt, s);
  store_row<N>(dA, mat, batch, r, dt);
}

// ------------------------------------------------ generator fused with Pade
// CGHC's transition Phi = exp(A) straight from the module's pre-activations
// (cghc.py:219-321), for a block of kExpmThreads / G tokens. One thread per
// token assembles A with the generator's own device code (generator.cuh) into
// shared memory; then G lanes per token run the Pade [7/7] evaluation on its
// rows exactly as expm_pade_fwd_kernel does on A read from global memory. The
// result is bit for bit that of the two launches, without A's round trip
// through HBM and one launch fewer.
template <int N, bool VEC>
__global__ void __launch_bounds__(kExpmThreads) transition_fwd_kernel(const GenArgs a, int flags,
                                                                      float* __restrict__ E) {
  constexpr int G = Group<N>::G;
  constexpr int MPB = kExpmThreads / G;
  __shared__ float sA[MPB * N * N];
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * MPB;
  if (threadIdx.x < MPB) {
    const int64_t t = t0 + threadIdx.x;
    float A[N * N];
    if (t < a.T) {
      gen_forward_token<N, VEC>(a, flags, t, A);
    } else {
#pragma unroll
      for (int k = 0; k < N * N; ++k) A[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < N * N; ++k) sA[threadIdx.x * N * N + k] = A[k];
  }
  __syncthreads();
  const int lm = threadIdx.x / G;
  const int r = threadIdx.x & (G - 1);
  const int64_t mat = t0 + lm;
  const bool ok = mat < a.T && r < N;
  float row[N];
#pragma unroll
  for (int j = 0; j < N; ++j) row[j] = ok ? sA[lm * N * N + r * N + j] : 0.f;
  const int s = scaling_exponent(norm1_rows<N, G>(row), kTheta7);
  const float sc = pow2_neg(s);
#pragma unroll
  for (int j = 0; j < N; ++j) row[j] *= sc;
  float t[N];
  pade7_eval<N, G>(row, r, t);
  square_s<N, G>(t, s);
  store_row<N>(E, mat, a.T, r, t);
}

// Backward of the same: A is assembled again (cheaper than storing it), the
// Pade Frechet backward of expm_pade_bwd_kernel gives dL/dA per row into
// shared memory, and one thread per token runs the generator's reverse mode
// on it. a.G is dL/dPhi here.
template <int N, bool VEC>
__global__ void __launch_bounds__(kExpmThreads) transition_bwd_kernel(const GenArgs a, int flags) {
  constexpr int G = Group<N>::G;
  constexpr int MPB = kExpmThreads / G;
  __shared__ float sA[MPB * N * N];
  __shared__ float sD[MPB * N * N];
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * MPB;
  if (threadIdx.x < MPB) {
    const int64_t t = t0 + threadIdx.x;
    float A[N * N];
    if (t < a.T) {
      gen_forward_token<N, VEC>(a, flags, t, A);
    } else {
#pragma unroll
      for (int k = 0; k < N * N; ++k) A[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < N * N; ++k) sA[threadIdx.x * N * N + k] = A[k];
  }
  __syncthreads();
  const int lm = threadIdx.x / G;
  const int r = threadIdx.x & (G - 1);
  const int64_t mat = t0 + lm;
  const bool ok = mat < a.T && r < N;
  float at[N], e[N];
#pragma unroll
  for (int j = 0; j < N; ++j) at[j] = ok ? sA[lm * N * N + j * N + r] : 0.f;  // row r of A^T
  load_row<N>(a.G, mat, a.T, r, e);
  const int s = scaling_exponent(norm1_from_transpose<N, G>(at), kTheta7);
  const float sc = pow2_neg(s);
#pragma unroll
  for (int j = 0; j < N; ++j) { at[j] *= sc; e[j] *= sc; }
  float t[N], dt[N];
  pade7_eval_d<N, G>(at, e, r, t, dt);
  square_s_d<N, G>(t, dt, s);
  if (ok) {
#pragma unroll
    for (int j = 0; j < N; ++j) sD[lm * N * N + r * N + j] = dt[j];
  }
  __syncthreads();
  if (threadIdx.x < MPB && t0 + threadIdx.x < a.T) {
    float dA[N * N];
#pragma unroll
    for (int k = 0; k < N * N; ++k) dA[k] = sD[threadIdx.x * N * N + k];
    gen_backward_token<N, VEC>(a, flags, t0 + threadIdx.x, dA);
  }
}

// ------------------------------------------------------------ host side
constexpr int kMaxNormParts = 1024;

int norm_parts(int64_t batch, int n) {
  const int G = n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8;
  const int64_t per_cta = kExpmThreads / G;
  int64_t parts = (batch + per_cta - 1) / per_cta;
  if (parts > kMaxNormParts) parts = kMaxNormParts;
  if (parts < 1) parts = 1;
  return static_cast<int>(parts);
}

dim3 expm_grid(int64_t batch, int n) {
  const int G = n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8;
  const int64_t threads = batch * G;
  return dim3(static_cast<unsigned>((threads + kExpmThreads - 1) / kExpmThreads), 1, 1);
}

int check(const void* a, const void* b, int64_t batch, int n) {
  if (batch < 0) return HC_ERR_BAD_SIZE;
  if (n < 1 || n > 8) return HC_ERR_UNSUPPORTED_N;
  // batch * 8 lanes / 256 threads per CTA must stay below 2^31 CTAs
  if (batch > (int64_t(1) << 34)) return HC_ERR_BAD_SIZE;
  if (batch == 0) return HC_OK;
  if (!a || !b) return HC_ERR_NULL_POINTER;
  if (!aligned4(a) || !aligned4(b)) return HC_ERR_ALIGNMENT;
  return HC_OK;
}

#define HC_EXPM_SWITCH(n, LAUNCH) \
  switch (n) {                    \
    case 1: LAUNCH(1); break;     \
    case 2: LAUNCH(2); break;     \
    case 3: LAUNCH(3); break;     \
    case 4: LAUNCH(4); break;     \
    case 5: LAUNCH(5); break;     \
    case 6: LAUNCH(6); break;     \
    case 7: LAUNCH(7); break;     \
    case 8: LAUNCH(8); break;     \
    default: return HC_ERR_UNSUPPORTED_N; \
  }

int launch_norm_partials(const float* A, int64_t batch, int n, float* scratch, int parts, cudaStream_t st) {
#define L(NN) expm_norm_partial_kernel<NN><<<parts, kExpmThreads, 0, st>>>(A, batch, scratch)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

// ---- the thread-per-matrix forward (n <= 4)
// Its global-scaling launch is cooperative: at most the CTAs that can be
// resident at once (occupancy x SMs), and at most kMaxNormParts - 1 of them
// so that the partials and the barrier counter fit the scratch of the
// two-kernel path. The partial maxima it leaves (one per CTA) are the ones
// hc_expm_t18_bwd mode 2 reads, so both use t18_parts().
constexpr int kTmMaxN = 4;

template <int N>
int tm_blocks_per_sm() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    cudaGetLastError();
    return 0;
  }
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, expm_t18_tm_coop_kernel<N>, kExpmThreads, 0) !=
          cudaSuccess ||
      nb <= 0) {
    cudaGetLastError();
    return 0;
  }
  if (dev < 64) cached[dev] = nb;
  return nb;
}

int tm_coop_grid(int64_t batch, int n) {
  int nb = 0;
  switch (n) {
    case 1: nb = tm_blocks_per_sm<1>(); break;
    case 2: nb = tm_blocks_per_sm<2>(); break;
    case 3: nb = tm_blocks_per_sm<3>(); break;
    default: nb = tm_blocks_per_sm<4>(); break;
  }
  if (nb <= 0) nb = 1;  // no device to ask (CPU-only process): a grid of SMs
  int64_t grid = (batch + kExpmThreads - 1) / kExpmThreads;
  grid = std::min<int64_t>(grid, static_cast<int64_t>(nb) * sm_count());
  grid = std::min<int64_t>(grid, kMaxNormParts - 1);
  return static_cast<int>(std::max<int64_t>(grid, 1));
}

// Partial maxima of the global-scaling forward (and of the backward's norm
// pass): one per CTA of the cooperative forward for n <= 4, one per CTA of
// the norm kernel otherwise.
int t18_parts(int64_t batch, int n) { return n <= kTmMaxN ? tm_coop_grid(batch, n) : norm_parts(batch, n); }

// Scratch words: the partials, plus the barrier counter of the cooperative
// launch for n <= 4.
int64_t t18_scratch_words(int64_t batch, int n) { return t18_parts(batch, n) + (n <= kTmMaxN ? 1 : 0); }

template <int N>
int launch_tm_fwd(const float* A, float* E, int64_t batch, float* scratch, int parts, bool global, cudaStream_t st) {
  const int vec = aligned16(A) && aligned16(E) ? 1 : 0;
  const int64_t full_grid = (batch + kExpmThreads - 1) / kExpmThreads;
  if (!global) {
    expm_t18_tm_fwd_kernel<N><<<static_cast<unsigned>(full_grid), kExpmThreads, 0, st>>>(A, E, batch, nullptr, 0,
                                                                                        vec);
    return launch_status();
  }
  if (full_grid > parts) {  // more matrices than resident threads: norm pass, then the grid-stride kernel
    if (int rc = launch_norm_partials(A, batch, N, scratch, parts, st)) return rc;
    expm_t18_tm_fwd_kernel<N><<<parts, kExpmThreads, 0, st>>>(A, E, batch, scratch, parts, vec);
    return launch_status();
  }
  unsigned int* arrive = reinterpret_cast<unsigned int*>(scratch + parts);
  if (cudaMemsetAsync(arrive, 0, sizeof(unsigned int), st) != cudaSuccess) {
    cudaGetLastError();
    return HC_ERR_LAUNCH;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(parts), 1, 1);
  cfg.blockDim = dim3(kExpmThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, expm_t18_tm_coop_kernel<N>, A, E, batch, scratch, arrive, vec,
                                           wait_poll_limit(), timeout_word(st));
  if (e == cudaErrorCooperativeLaunchTooLarge) {
    // fewer SMs usable than the device reports (an MPS share, for one): the
    // two-launch form needs no co-residency and writes the same partials
    cudaGetLastError();
    if (int rc = launch_norm_partials(A, batch, N, scratch, parts, st)) return rc;
    expm_t18_tm_fwd_kernel<N><<<parts, kExpmThreads, 0, st>>>(A, E, batch, scratch, parts, vec);
    return launch_status();
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return HC_ERR_LAUNCH;
  }
  return launch_status();
}

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int64_t hc_expm_t18_scratch_words(int64_t batch, int n) {
  if (batch < 0 || n < 1 || n > 8) return 0;
  return t18_scratch_words(batch, n);
}

extern "C" int hc_expm_t18_fwd(const float* A, float* E, int64_t batch, int n, float* scratch,
                               int64_t scratch_words, int per_matrix, void* stream) {
  HC_ENTRY("hc_expm_t18_fwd");
  if (per_matrix != 0 && per_matrix != 1) return HC_ERR_BAD_SIZE;
  int rc = check(A, E, batch, n);
  if (rc || batch == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n <= kTmMaxN) {
    int parts = 0;
    if (!per_matrix) {
      parts = t18_parts(batch, n);
      if (!scratch || scratch_words < t18_scratch_words(batch, n)) return HC_ERR_SCRATCH;
      if (!aligned4(scratch)) return HC_ERR_ALIGNMENT;
    }
    switch (n) {
      case 1: return launch_tm_fwd<1>(A, E, batch, scratch, parts, !per_matrix, st);
      case 2: return launch_tm_fwd<2>(A, E, batch, scratch, parts, !per_matrix, st);
      case 3: return launch_tm_fwd<3>(A, E, batch, scratch, parts, !per_matrix, st);
      default: return launch_tm_fwd<4>(A, E, batch, scratch, parts, !per_matrix, st);
    }
  }
  const float* partial = nullptr;
  int parts = 0;
  if (!per_matrix) {
    parts = t18_parts(batch, n);
    if (!scratch || scratch_words < t18_scratch_words(batch, n)) return HC_ERR_SCRATCH;
    if (!aligned4(scratch)) return HC_ERR_ALIGNMENT;
    rc = launch_norm_partials(A, batch, n, scratch, parts, st);
    if (rc) return rc;
    partial = scratch;
  }
  const dim3 grid = expm_grid(batch, n);
#define L(NN) expm_t18_fwd_kernel<NN><<<grid, kExpmThreads, 0, st>>>(A, E, batch, partial, parts)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

extern "C" int hc_expm_t18_bwd(const float* A, const float* G, float* dA, int64_t batch, int n,
                               float* scratch, int64_t scratch_words, int per_matrix, void* stream) {
  HC_ENTRY("hc_expm_t18_bwd");
  if (per_matrix < 0 || per_matrix > 2) return HC_ERR_BAD_SIZE;
  int rc = check(A, dA, batch, n);
  if (rc || batch == 0) return rc;
  if (!G) return HC_ERR_NULL_POINTER;
  if (!aligned4(G)) return HC_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* partial = nullptr;
  int parts = 0;
  if (per_matrix != 1) {
    parts = t18_parts(batch, n);
    if (!scratch || scratch_words < t18_scratch_words(batch, n)) return HC_ERR_SCRATCH;
    if (!aligned4(scratch)) return HC_ERR_ALIGNMENT;
    if (per_matrix == 0) {  // mode 2: the forward's partial maxima of this A are already in scratch
      rc = launch_norm_partials(A, batch, n, scratch, parts, st);
      if (rc) return rc;
    }
    partial = scratch;
  }
  if (n <= kTmMaxN) {
    const int vec = aligned16(A) && aligned16(G) && aligned16(dA) ? 1 : 0;
    const dim3 grid(static_cast<unsigned>((batch + kExpmTmBwdThreads - 1) / kExpmTmBwdThreads), 1, 1);
#define L(NN) \
  expm_t18_tm_bwd_kernel<NN><<<grid, kExpmTmBwdThreads, 0, st>>>(A, G, dA, batch, partial, parts, vec)
    switch (n) {
      case 1: L(1); break;
      case 2: L(2); break;
      case 3: L(3); break;
      default: L(4); break;
    }
#undef L
    return launch_status();
  }
  const dim3 grid = expm_grid(batch, n);
#define L(NN) expm_t18_bwd_kernel<NN><<<grid, kExpmThreads, 0, st>>>(A, G, dA, batch, partial, parts)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

extern "C" int hc_expm_pade_fwd(const float* A, float* E, int64_t batch, int n, void* stream) {
  HC_ENTRY("hc_expm_pade_fwd");
  int rc = check(A, E, batch, n);
  if (rc || batch == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid = expm_grid(batch, n);
#define L(NN) expm_pade_fwd_kernel<NN><<<grid, kExpmThreads, 0, st>>>(A, E, batch)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

extern "C" int hc_expm_pade_bwd(const float* A, const float* G, float* dA, int64_t batch, int n,
                                void* stream) {
  HC_ENTRY("hc_expm_pade_bwd");
  int rc = check(A, dA, batch, n);
  if (rc || batch == 0) return rc;
  if (!G) return HC_ERR_NULL_POINTER;
  if (!aligned4(G)) return HC_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid = expm_grid(batch, n);
#define L(NN) expm_pade_bwd_kernel<NN><<<grid, kExpmThreads, 0, st>>>(A, G, dA, batch)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

namespace hc {
namespace {

int check_transition(const GenArgs& a, int n, int flags) {
  if (a.T > (int64_t(1) << 34)) return HC_ERR_BAD_SIZE;  // T / 32 tokens per CTA stays below 2^31 CTAs
  return check_gen(a, n, flags);
}

unsigned transition_grid(int64_t T, int n) {
  const int G = n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : 8;
  const int64_t per_cta = kExpmThreads / G;
  return static_cast<unsigned>((T + per_cta - 1) / per_cta);
}

}  // namespace
}  // namespace hc

extern "C" int hc_cghc_transition_fwd(const float* M, const float* lc, const float* R, const float* dpre,
                                      const float* S, const float* ld, float* Phi, int64_t T, int n, int vec_dt,
                                      int flags, float dt_min_c, float dt_max_c, float dt_min_d, float dt_max_d,
                                      void* stream) {
  HC_ENTRY("hc_cghc_transition_fwd");
  GenArgs a{};
  a.M = M; a.lc = lc; a.ld = ld; a.R = R; a.dpre = dpre; a.S = S; a.T = T;
  a.lo_c = dt_min_c; a.hi_c = dt_max_c; a.lo_d = dt_min_d; a.hi_d = dt_max_d;
  int rc = check_transition(a, n, flags);
  if (rc || T == 0) return rc;
  if (!Phi) return HC_ERR_NULL_POINTER;
  if (!aligned4(Phi)) return HC_ERR_ALIGNMENT;
  const unsigned grid = transition_grid(T, n);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define L(NN)                                                                                  \
  if (vec_dt) transition_fwd_kernel<NN, true><<<grid, kExpmThreads, 0, st>>>(a, flags, Phi);  \
  else transition_fwd_kernel<NN, false><<<grid, kExpmThreads, 0, st>>>(a, flags, Phi)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

extern "C" int hc_cghc_transition_bwd(const float* M, const float* lc, const float* R, const float* dpre,
                                      const float* S, const float* ld, const float* G, float* dM, float* dlc,
                                      float* dR, float* ddpre, float* dS, float* dld, int64_t T, int n, int vec_dt,
                                      int flags, float dt_min_c, float dt_max_c, float dt_min_d, float dt_max_d,
                                      void* stream) {
  HC_ENTRY("hc_cghc_transition_bwd");
  GenArgs a{};
  a.M = M; a.lc = lc; a.ld = ld; a.R = R; a.dpre = dpre; a.S = S; a.G = G; a.T = T;
  a.dM = dM; a.dlc = dlc; a.dld = dld; a.dR = dR; a.ddpre = ddpre; a.dS = dS;
  a.lo_c = dt_min_c; a.hi_c = dt_max_c; a.lo_d = dt_min_d; a.hi_d = dt_max_d;
  int rc = check_transition(a, n, flags);
  if (rc || T == 0) return rc;
  if (!G) return HC_ERR_NULL_POINTER;
  const unsigned grid = transition_grid(T, n);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define L(NN)                                                                           \
  if (vec_dt) transition_bwd_kernel<NN, true><<<grid, kExpmThreads, 0, st>>>(a, flags);  \
  else transition_bwd_kernel<NN, false><<<grid, kExpmThreads, 0, st>>>(a, flags)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

// ------------------------------------------------------------ no-allocation variant
// Some callers cannot allocate device memory at all: a plugin or FFI caller
// that only ever receives pointers from a host framework which owns every
// byte of device memory, or a latency-critical loop that must not call
// cudaMalloc because it can synchronise the whole device. For them,
// hc_expm_t18_fwd_noalloc keeps the global-scaling scratch (one partial
// maximum of ||A||_1 per CTA of the norm kernel) in this fixed array instead
// of a caller buffer. Every GPU that loads the library holds these 4 KB until
// the process exits.
namespace hc {
namespace {

constexpr int kNoallocMaxDevices = 64;
static __device__ __align__(256) float g_t18_noalloc_partials[kMaxNormParts];

std::mutex g_noalloc_mu;
float* g_noalloc_dev_ptr[kNoallocMaxDevices] = {};

// Device address of the array on the current device, looked up once per
// device (the array's name in host code is only a host-side stand-in).
int noalloc_scratch(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return HC_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kNoallocMaxDevices) return HC_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_dev_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_t18_noalloc_partials);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return HC_ERR_LAUNCH;
    }
    g_noalloc_dev_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_dev_ptr[dev];
  return HC_OK;
}

}  // namespace
}  // namespace hc

extern "C" int hc_expm_t18_fwd_noalloc(const float* A, float* E, int64_t batch, int n, void* stream) {
  int rc = check(A, E, batch, n);
  if (rc || batch == 0) return rc;
  // norm_parts() caps the partial maxima at kMaxNormParts (the norm kernel
  // strides over the batch), the size of the array: any batch up to the
  // 2^34-matrix bound fits.
  const int parts = norm_parts(batch, n);
  float* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Every slot the expm kernel reads (0 .. parts-1) is written first by the
  // norm kernel of this same call, so nothing needs clearing beforehand.
  rc = launch_norm_partials(A, batch, n, scratch, parts, st);
  if (rc) return rc;
  const dim3 grid = expm_grid(batch, n);
#define L(NN) expm_t18_fwd_kernel<NN><<<grid, kExpmThreads, 0, st>>>(A, E, batch, scratch, parts)
  HC_EXPM_SWITCH(n, L)
#undef L
  return launch_status();
}

namespace hc {
unsigned int expm_take_timeouts(bool reset) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_expm_wait_timeouts, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (reset && v != 0) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_expm_wait_timeouts, &z, sizeof(z));
  }
  return v;
}
}  // namespace hc
