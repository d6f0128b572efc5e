// sinkhorn.cu — batched Sinkhorn-Knopp projection of small matrices (n <= 8),
// forward and backward, float32.
//
// Per matrix (reference hyperconnections/mhc.py:97-102, _sinkhorn_knopp):
//   X_0 = exp(H)
//   for k = 1..iters:  Y_k = X_{k-1} / rowsum(X_{k-1})     (each row sums to 1)
//                      X_k = Y_k / colsum(Y_k)             (each column sums to 1)
//   P = X_iters
// Backward, given G = dL/dP, in reverse order of the steps:
//   column step   dY_ij = (dX_ij - sum_l dX_lj X_lj) / c_j,  X_lj = Y_lj / c_j
//   row step      dX_ij = (dY_ij - sum_l dY_il Y_il) / r_i
//   exp           dH = dX_0 * X_0
// (the autograd rules of the reference's divisions and sums, applied per step).
//
// A group of lanes owns a matrix, one row per lane (column sums by shuffles);
// a CTA stages its matrices through shared memory so that global loads and
// stores are coalesced. Up to kSkLinearIters iterations the backward keeps
// the row and column sums of every iteration and rebuilds the iterates in
// reverse (linear time); beyond that one thread per matrix recomputes the
// forward prefix X_{k-1} for each step k from X_0 (iters^2 / 2 half-steps,
// no stored iterates).
#include "common.cuh"

namespace hc {
namespace {

constexpr int kSkThreads = 128;
constexpr int kSkMaxIters = 256;

template <int N>
__device__ __forceinline__ void row_normalize(float* x, float* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < N; ++j) s += x[i * N + j];
    r[i] = s;
#pragma unroll
    for (int j = 0; j < N; ++j) x[i * N + j] = x[i * N + j] / s;
  }
}

template <int N>
__device__ __forceinline__ void col_normalize(float* x, float* c) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) s += x[i * N + j];
    c[j] = s;
#pragma unroll
    for (int i = 0; i < N; ++i) x[i * N + j] = x[i * N + j] / s;
  }
}

// Shared-memory row of one matrix: N*N floats plus one pad word, so that the
// threads of a warp (consecutive matrices) fall into different banks.
template <int N> constexpr int sk_pitch() { return N * N + 1; }

template <int N>
__device__ __forceinline__ void stage_in(const float* __restrict__ g, float* sm, int64_t first, int cnt) {
  const float* src = g + first * (N * N);
  for (int i = threadIdx.x; i < cnt * N * N; i += blockDim.x) sm[(i / (N * N)) * sk_pitch<N>() + i % (N * N)] = src[i];
}

template <int N>
__device__ __forceinline__ void stage_out(float* __restrict__ g, const float* sm, int64_t first, int cnt) {
  float* dst = g + first * (N * N);
  for (int i = threadIdx.x; i < cnt * N * N; i += blockDim.x) dst[i] = sm[(i / (N * N)) * sk_pitch<N>() + i % (N * N)];
}

template <int N>
__global__ void __launch_bounds__(kSkThreads) sinkhorn_bwd_kernel(const float* __restrict__ H,
                                                                  const float* __restrict__ G,
                                                                  float* __restrict__ dH, int64_t batch, int iters) {
  __shared__ float sm[kSkThreads * sk_pitch<N>()];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kSkThreads;
  const int cnt = static_cast<int>(batch - first < kSkThreads ? batch - first : kSkThreads);
  float x0[N * N], g[N * N];
  stage_in<N>(H, sm, first, cnt);
  __syncthreads();
  float* row = sm + threadIdx.x * sk_pitch<N>();
  if (threadIdx.x < cnt) {
#pragma unroll
    for (int k = 0; k < N * N; ++k) x0[k] = expf(row[k]);
  }
  __syncthreads();
  stage_in<N>(G, sm, first, cnt);
  __syncthreads();
  if (threadIdx.x < cnt) {
#pragma unroll
    for (int k = 0; k < N * N; ++k) g[k] = row[k];
    for (int k = iters; k >= 1; --k) {
      float y[N * N], r[N], c[N];
#pragma unroll
      for (int q = 0; q < N * N; ++q) y[q] = x0[q];
      for (int it = 1; it < k; ++it) {  // X_{k-1}
        row_normalize<N>(y, r);
        col_normalize<N>(y, c);
      }
      row_normalize<N>(y, r);  // Y_k and its row sums r
#pragma unroll
      for (int j = 0; j < N; ++j) {  // column sums of Y_k
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) s += y[i * N + j];
        c[j] = s;
      }
      // column step: dY_ij = (g_ij - sum_l g_lj X_lj) / c_j with X_lj = Y_lj / c_j
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float t = 0.f;
#pragma unroll
        for (int l = 0; l < N; ++l) t += g[l * N + j] * (y[l * N + j] / c[j]);
#pragma unroll
        for (int i = 0; i < N; ++i) g[i * N + j] = (g[i * N + j] - t) / c[j];
      }
      // row step: dX_ij = (dY_ij - sum_l dY_il Y_il) / r_i
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float t = 0.f;
#pragma unroll
        for (int l = 0; l < N; ++l) t += g[i * N + l] * y[i * N + l];
#pragma unroll
        for (int j = 0; j < N; ++j) g[i * N + j] = (g[i * N + j] - t) / r[i];
      }
    }
#pragma unroll
    for (int q = 0; q < N * N; ++q) row[q] = g[q] * x0[q];
  }
  __syncthreads();
  stage_out<N>(dH, sm, first, cnt);
}

// Backward in linear time for iters <= kSkLinearIters: the forward is run
// once, keeping every iteration's row sums r_k and column sums c_k (in local
// memory); the backward then walks the steps in reverse, rebuilding the
// iterates from the final X by multiplication, Y_k = X_k c_k (columns) and
// X_{k-1} = Y_k r_k (rows), instead of recomputing each prefix from X_0. The
// rebuilt iterates differ from the forward's by a few units in the last place
// after 20 iterations, far inside fp32 gradient accuracy; X_iters itself and
// X_0 = exp(H) are exact.
constexpr int kSkLinearIters = 32;

// ------------------------------------------------ one lane per row
// A group of G lanes (G = n rounded up to a power of two) owns a matrix, lane
// r its row r: a row sum is local, a column sum a log2(G)-step xor-shuffle
// tree across the group. n to 8 times the threads of one thread per matrix,
// and an n times shorter chain of divisions per thread. Lanes r >= n keep a
// zero row and skip the row division (no 0/0); their column contributions
// are zeros. The shuffles run on all 32 lanes, so lanes without a matrix
// (past the batch) compute on a zero-filled copy and store nothing.
template <int N> struct SkGroup {
  static constexpr int G = N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : 8;
  static constexpr int kMats = kSkThreads / G;  // matrices per CTA
};

template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = 1; o < G; o <<= 1) v += __shfl_xor_sync(kFull, v, o, G);
  return v;
}

// Row r of matrix (first + m) from the CTA's staged copy, zeros outside.
template <int N>
__device__ __forceinline__ void sk_row_in(const float* sm, int m, int r, int cnt, float (&v)[N]) {
  const bool ok = m < cnt && r < N;
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] = ok ? sm[m * sk_pitch<N>() + r * N + j] : 0.f;
}

template <int N>
__device__ __forceinline__ void sk_row_out(float* sm, int m, int r, int cnt, const float (&v)[N]) {
  if (m >= cnt || r >= N) return;
#pragma unroll
  for (int j = 0; j < N; ++j) sm[m * sk_pitch<N>() + r * N + j] = v[j];
}

// One Sinkhorn iteration on this lane's row; returns the row sum and the
// column sums (every lane of the group gets all of them).
template <int N, int G>
__device__ __forceinline__ float sk_iter_row(float (&x)[N], bool real_row, float (&c)[N]) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < N; ++j) s += x[j];
  if (real_row) {
#pragma unroll
    for (int j = 0; j < N; ++j) x[j] = x[j] / s;
  }
#pragma unroll
  for (int j = 0; j < N; ++j) {
    c[j] = group_sum<G>(x[j]);
    x[j] = x[j] / c[j];
  }
  return s;
}

template <int N>
__global__ void __launch_bounds__(kSkThreads) sinkhorn_fwd_rows_kernel(const float* __restrict__ H,
                                                                       float* __restrict__ P, int64_t batch,
                                                                       int iters) {
  constexpr int G = SkGroup<N>::G, M = SkGroup<N>::kMats;
  __shared__ float sm[M * sk_pitch<N>()];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * M;
  const int cnt = static_cast<int>(batch - first < M ? batch - first : M);
  stage_in<N>(H, sm, first, cnt);
  __syncthreads();
  const int m = threadIdx.x / G, r = threadIdx.x % G;
  const bool real_row = m < cnt && r < N;
  float x[N];
  sk_row_in<N>(sm, m, r, cnt, x);
#pragma unroll
  for (int j = 0; j < N; ++j) x[j] = real_row ? expf(x[j]) : 0.f;
  for (int it = 0; it < iters; ++it) {
    float c[N];
    sk_iter_row<N, G>(x, real_row, c);
  }
  __syncthreads();
  sk_row_out<N>(sm, m, r, cnt, x);
  __syncthreads();
  stage_out<N>(P, sm, first, cnt);
}

// Linear-time backward (iters <= kSkLinearIters) in the row-per-lane layout:
// the forward keeps this lane's row sum and all column sums per iteration.
template <int N>
__global__ void __launch_bounds__(kSkThreads) sinkhorn_bwd_rows_kernel(const float* __restrict__ H,
                                                                       const float* __restrict__ Gr,
                                                                       float* __restrict__ dH, int64_t batch,
                                                                       int iters) {
  constexpr int G = SkGroup<N>::G, M = SkGroup<N>::kMats;
  __shared__ float sm[M * sk_pitch<N>()];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * M;
  const int cnt = static_cast<int>(batch - first < M ? batch - first : M);
  const int m = threadIdx.x / G, r = threadIdx.x % G;
  const bool real_row = m < cnt && r < N;
  float x0[N], g[N];
  stage_in<N>(H, sm, first, cnt);
  __syncthreads();
  sk_row_in<N>(sm, m, r, cnt, x0);
#pragma unroll
  for (int j = 0; j < N; ++j) x0[j] = real_row ? expf(x0[j]) : 0.f;
  __syncthreads();
  stage_in<N>(Gr, sm, first, cnt);
  __syncthreads();
  sk_row_in<N>(sm, m, r, cnt, g);
  float rs[kSkLinearIters], cs[kSkLinearIters][N];
  float x[N];
#pragma unroll
  for (int j = 0; j < N; ++j) x[j] = x0[j];
  for (int it = 0; it < iters; ++it) {
    float c[N];
    rs[it] = sk_iter_row<N, G>(x, real_row, c);
#pragma unroll
    for (int j = 0; j < N; ++j) cs[it][j] = c[j];
  }
  for (int k = iters - 1; k >= 0; --k) {  // x holds row r of X_{k+1}
    const float rr = real_row ? rs[k] : 1.f;
    float c[N], y[N];
#pragma unroll
    for (int j = 0; j < N; ++j) c[j] = cs[k][j];
    // column step: dY_ij = (g_ij - sum_l g_lj X_lj) / c_j
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float t = group_sum<G>(g[j] * x[j]);
      g[j] = real_row ? (g[j] - t) / c[j] : 0.f;
      y[j] = x[j] * c[j];
    }
    // row step: dX_ij = (dY_ij - sum_l dY_il Y_il) / r_i
    float t = 0.f;
#pragma unroll
    for (int l = 0; l < N; ++l) t += g[l] * y[l];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      g[j] = (g[j] - t) / rr;
      x[j] = y[j] * rr;
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) g[j] *= x0[j];
  __syncthreads();
  sk_row_out<N>(sm, m, r, cnt, g);
  __syncthreads();
  stage_out<N>(dH, sm, first, cnt);
}

unsigned rows_grid(int64_t batch, int mats_per_cta) {
  return static_cast<unsigned>((batch + mats_per_cta - 1) / mats_per_cta);
}

int check_sk(const void* a, const void* b, int64_t batch, int n, int iters) {
  if (batch < 0 || batch > (int64_t(1) << 37)) return HC_ERR_BAD_SIZE;
  if (iters < 0 || iters > kSkMaxIters) return HC_ERR_BAD_SIZE;
  if (n < 1 || n > 8) return HC_ERR_UNSUPPORTED_N;
  if (batch == 0) return HC_OK;
  if (!a || !b) return HC_ERR_NULL_POINTER;
  if (!aligned4(a) || !aligned4(b)) return HC_ERR_ALIGNMENT;
  return HC_OK;
}

#define HC_SK_SWITCH(n, LAUNCH) \
  switch (n) {                  \
    case 1: LAUNCH(1); break;   \
    case 2: LAUNCH(2); break;   \
    case 3: LAUNCH(3); break;   \
    case 4: LAUNCH(4); break;   \
    case 5: LAUNCH(5); break;   \
    case 6: LAUNCH(6); break;   \
    case 7: LAUNCH(7); break;   \
    case 8: LAUNCH(8); break;   \
    default: return HC_ERR_UNSUPPORTED_N; \
  }

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_sinkhorn_fwd(const float* H, float* P, int64_t batch, int n, int iters, void* stream) {
  HC_ENTRY("hc_sinkhorn_fwd");
  int rc = check_sk(H, P, batch, n, iters);
  if (rc || batch == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define L(NN)                                                                                   \
  sinkhorn_fwd_rows_kernel<NN><<<rows_grid(batch, SkGroup<NN>::kMats), kSkThreads, 0, st>>>(H, P, batch, \
                                                                                            iters)
  HC_SK_SWITCH(n, L)
#undef L
  return launch_status();
}

extern "C" int hc_sinkhorn_bwd(const float* H, const float* G, float* dH, int64_t batch, int n, int iters,
                               void* stream) {
  HC_ENTRY("hc_sinkhorn_bwd");
  int rc = check_sk(H, dH, batch, n, iters);
  if (rc || batch == 0) return rc;
  if (!G) return HC_ERR_NULL_POINTER;
  if (!aligned4(G)) return HC_ERR_ALIGNMENT;
  const unsigned grid = static_cast<unsigned>((batch + kSkThreads - 1) / kSkThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (iters <= kSkLinearIters) {
#define L(NN)                                                                                        \
  sinkhorn_bwd_rows_kernel<NN><<<rows_grid(batch, SkGroup<NN>::kMats), kSkThreads, 0, st>>>(H, G, dH, batch, \
                                                                                             iters)
    HC_SK_SWITCH(n, L)
#undef L
    return launch_status();
  }
#define L(NN) sinkhorn_bwd_kernel<NN><<<grid, kSkThreads, 0, st>>>(H, G, dH, batch, iters)
  HC_SK_SWITCH(n, L)
#undef L
  return launch_status();
}
