// mix_kernels.cuh — per-token stream-mixing kernels (forward and backward).
//
// One "token" is the n x D block of stream state of one (batch, position).
// Every token is independent, so the grid is a 2-D tile of
//   blockDim.x = TX threads over the D-chunks of a token (TX multiple of 32),
//   blockDim.y = TY tokens per CTA,
// and each thread walks chunks c = threadIdx.x + p*TX, p < passes. A thread
// loads the chunk of ALL n streams at once (n 16-byte loads), so every byte of
// the stream state is read from HBM exactly once and written exactly once.
//
// Two modes share the code:
//   FUSED = false  (stream_mix_add, reference ops/stream_mix_small_nb.py:75-132)
//       out_i = sum_j Phi_ij x_j  [+ (v_i - (Phi v)_i) (v^T x)]  + Y_i
//   FUSED = true   (width-read + mix + depth-write, m = 1;
//                   reference cghc.py:410, :417, :449)
//       u      = sum_j alpha_j x_j
//       out_i  = sum_j H_ij x_j + beta_i f
//
// The backward kernels also reduce the per-token parameter gradients over D
// (grad_Phi / grad_H, grad_alpha, grad_beta, and the projection terms): each
// thread accumulates its partial sums in registers, a warp transpose-reduce
// folds 32 lanes, and a shared-memory pass folds the TX/32 warps of a token.
// One CTA owns whole tokens, so no atomics and no global scratch are needed.
#pragma once

#include "common.cuh"

namespace hc {

struct MixFwdArgs {
  const void* x;      // [T,N,D]
  const void* src;    // Y [T,N,D] (add) | f [T,D] (fused)
  const void* phi;    // [T,N,N]  P
  const void* v;      // [T,N]    P   (projection; add mode only)
  const float* alpha; // [T,N]        (fused)
  const float* beta;  // [T,N]        (fused)
  void* out;          // [T,N,D]
  void* u;            // [T,D]        (fused)
  int64_t T;
  int64_t D;
  int nchunk;         // chunks per stream row
  int passes;         // ceil(nchunk / blockDim.x)
};

struct MixBwdArgs {
  const void* g;      // dL/dout [T,N,D]
  const void* gu;     // dL/du   [T,D]  (fused)
  const void* x;      // [T,N,D]
  const void* f;      // [T,D]          (fused)
  const void* phi;    // [T,N,N] P
  const void* v;      // [T,N]   P      (projection)
  const float* alpha; // [T,N]          (fused)
  const float* beta;  // [T,N]          (fused)
  void* grad_x;       // [T,N,D]        nullable
  void* grad_f;       // [T,D]          nullable (fused)
  float* grad_phi;    // [T,N,N]        nullable
  float* grad_v;      // [T,N]          nullable (projection)
  float* grad_alpha;  // [T,N]          nullable (fused)
  float* grad_beta;   // [T,N]          nullable (fused)
  int64_t T;
  int64_t D;
  int nchunk;
  int passes;
};

constexpr int kMaxCtaThreads = 256;

// ============================================================== forward
template <typename T, typename P, int N, bool FUSED, bool PROJ, bool VECTOR>
__global__ void __launch_bounds__(kMaxCtaThreads)
mix_fwd_kernel(const MixFwdArgs a) {
  using C = Chunk<T, VECTOR>;
  constexpr int E = C::E;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  if (t >= a.T) return;  // no block-wide barrier in the forward

  float phi[N * N];
  load_params<P, N * N>(static_cast<const P*>(a.phi) + t * (N * N), phi);

  float vv[N], cc[N];  // projection direction and c = v - Phi v
  if constexpr (PROJ) {
    load_params<P, N>(static_cast<const P*>(a.v) + t * N, vv);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float pv = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) pv = fmaf(phi[i * N + j], vv[j], pv);
      cc[i] = vv[i] - pv;
    }
  }
  float al[N], be[N];
  if constexpr (FUSED) {
    load_params<float, N>(a.alpha + t * N, al);
    load_params<float, N>(a.beta + t * N, be);
  }

  const int64_t D = a.D;
  const T* __restrict__ xt = static_cast<const T*>(a.x) + t * N * D;
  T* __restrict__ ot = static_cast<T*>(a.out) + t * N * D;
  const T* __restrict__ st = static_cast<const T*>(a.src) + (FUSED ? t * D : t * N * D);
  T* __restrict__ ut = FUSED ? static_cast<T*>(a.u) + t * D : nullptr;

  for (int p = 0; p < a.passes; ++p) {
    const int ch = threadIdx.x + p * blockDim.x;
    const bool ok = ch < a.nchunk;
    const int64_t off = static_cast<int64_t>(ch) * E;

    float xv[N][E];
#pragma unroll
    for (int j = 0; j < N; ++j) C::load(xt + j * D + off, ok, xv[j]);
    constexpr int NS = FUSED ? 1 : N;
    float sv[NS][E];
#pragma unroll
    for (int i = 0; i < NS; ++i) C::load(st + i * D + off, ok, sv[i]);
    if (!ok) break;

    float av[E];  // v^T x per element (projection)
    if constexpr (PROJ) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) s = fmaf(vv[j], xv[j][e], s);
        av[e] = s;
      }
    }
    if constexpr (FUSED) {
      float uo[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) s = fmaf(al[j], xv[j][e], s);
        uo[e] = s;
      }
      C::store(ut + off, true, uo);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float o[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) s = fmaf(phi[i * N + j], xv[j][e], s);
        if constexpr (PROJ) s = fmaf(cc[i], av[e], s);
        if constexpr (FUSED) {
          s = fmaf(be[i], sv[0][e], s);
        } else {
          s = s + sv[i][e];
        }
        o[e] = s;
      }
      C::store(ot + i * D + off, true, o);
    }
  }
}

// ============================================================== backward
template <int N, bool FUSED, bool PROJ>
struct BwdLayout {
  // accumulator slots: [0, N*N) grad_phi(i,j); then
  //   FUSED: [N*N, N*N+N) grad_alpha_j, [N*N+N, N*N+2N) grad_beta_i
  //   PROJ : [N*N, N*N+N) rho_i,        [N*N+N, N*N+2N) beta-part_j
  static constexpr int kAcc = N * N + ((FUSED || PROJ) ? 2 * N : 0);
  static constexpr int kR = (kAcc + 31) / 32;  // values per lane after reduce
  static constexpr int kPad = 32 * kR;
};

template <typename T, typename P, int N, bool FUSED, bool PROJ, bool VECTOR>
__global__ void __launch_bounds__(kMaxCtaThreads)
mix_bwd_kernel(const MixBwdArgs a) {
  using C = Chunk<T, VECTOR>;
  using L = BwdLayout<N, FUSED, PROJ>;
  constexpr int E = C::E;
  constexpr int R = L::kR;

  __shared__ float red[kMaxCtaThreads / 32][L::kPad];
  __shared__ float fin[PROJ ? kMaxCtaThreads / 32 : 1][PROJ ? L::kAcc : 1];

  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool tok_ok = t < a.T;
  const int64_t ts = tok_ok ? t : 0;  // safe index for parameter loads

  float phi[N * N];
  load_params<P, N * N>(static_cast<const P*>(a.phi) + ts * (N * N), phi);
  float vv[N], cc[N];
  if constexpr (PROJ) {
    load_params<P, N>(static_cast<const P*>(a.v) + ts * N, vv);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float pv = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) pv = fmaf(phi[i * N + j], vv[j], pv);
      cc[i] = vv[i] - pv;
    }
  }
  float al[N], be[N];
  if constexpr (FUSED) {
    load_params<float, N>(a.alpha + ts * N, al);
    load_params<float, N>(a.beta + ts * N, be);
  }

  float acc[L::kPad];
#pragma unroll
  for (int k = 0; k < L::kPad; ++k) acc[k] = 0.f;

  const int64_t D = a.D;
  const T* __restrict__ gt = static_cast<const T*>(a.g) + ts * N * D;
  const T* __restrict__ xt = static_cast<const T*>(a.x) + ts * N * D;
  const T* __restrict__ gut = FUSED ? static_cast<const T*>(a.gu) + ts * D : nullptr;
  const T* __restrict__ ft = FUSED ? static_cast<const T*>(a.f) + ts * D : nullptr;
  T* __restrict__ gxt = a.grad_x ? static_cast<T*>(a.grad_x) + ts * N * D : nullptr;
  T* __restrict__ gft = (FUSED && a.grad_f) ? static_cast<T*>(a.grad_f) + ts * D : nullptr;

  for (int p = 0; p < a.passes; ++p) {
    const int ch = threadIdx.x + p * blockDim.x;
    const bool ok = tok_ok && ch < a.nchunk;
    const int64_t off = static_cast<int64_t>(ch) * E;

    float gv[N][E], xv[N][E];
#pragma unroll
    for (int i = 0; i < N; ++i) C::load(gt + i * D + off, ok, gv[i]);
#pragma unroll
    for (int j = 0; j < N; ++j) C::load(xt + j * D + off, ok, xv[j]);
    float guv[E], fv[E];
    if constexpr (FUSED) {
      C::load(gut + off, ok, guv);
      C::load(ft + off, ok, fv);
    }

    float av[E], bt[E];  // v^T x and c^T g per element (projection)
    if constexpr (PROJ) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float s = 0.f, b = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) s = fmaf(vv[j], xv[j][e], s);
#pragma unroll
        for (int i = 0; i < N; ++i) b = fmaf(gv[i][e], cc[i], b);
        av[e] = s;
        bt[e] = b;
      }
    }

    // grad_x_j = sum_i Phi_ij g_i (+ v_j beta) (+ alpha_j g_u)
    if (gxt != nullptr) {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float o[E];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) s = fmaf(phi[i * N + j], gv[i][e], s);
          if constexpr (PROJ) s = fmaf(vv[j], bt[e], s);
          if constexpr (FUSED) s = fmaf(al[j], guv[e], s);
          o[e] = s;
        }
        C::store(gxt + j * D + off, ok, o);
      }
    }
    if constexpr (FUSED) {
      if (gft != nullptr) {
        float o[E];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) s = fmaf(be[i], gv[i][e], s);
          o[e] = s;
        }
        C::store(gft + off, ok, o);
      }
    }

    // per-token reductions over D
#pragma unroll
    for (int e = 0; e < E; ++e) {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float xe = xv[j][e];
        if constexpr (PROJ) xe = xe - vv[j] * av[e];  // x_eff = x - v (v^T x)
#pragma unroll
        for (int i = 0; i < N; ++i) acc[i * N + j] = fmaf(gv[i][e], xe, acc[i * N + j]);
      }
      if constexpr (FUSED) {
#pragma unroll
        for (int j = 0; j < N; ++j) acc[N * N + j] = fmaf(guv[e], xv[j][e], acc[N * N + j]);
#pragma unroll
        for (int i = 0; i < N; ++i) acc[N * N + N + i] = fmaf(gv[i][e], fv[e], acc[N * N + N + i]);
      }
      if constexpr (PROJ) {
#pragma unroll
        for (int i = 0; i < N; ++i) acc[N * N + i] = fmaf(gv[i][e], av[e], acc[N * N + i]);
#pragma unroll
        for (int j = 0; j < N; ++j) acc[N * N + N + j] = fmaf(bt[e], xv[j][e], acc[N * N + N + j]);
      }
    }
  }

  // ---- fold the partial sums of the token's TX threads
  const int lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;                      // warps per token
  const int wid = threadIdx.y * nw + (threadIdx.x >> 5);  // warp in CTA
  warp_transpose_reduce<R>(acc, lane);
#pragma unroll
  for (int r = 0; r < R; ++r) red[wid][lane * R + r] = acc[r];
  __syncthreads();

  if (tok_ok) {
    for (int k = threadIdx.x; k < L::kAcc; k += blockDim.x) {
      float s = 0.f;
      for (int w = 0; w < nw; ++w) s += red[threadIdx.y * nw + w][k];
      if (k < N * N) {
        if (a.grad_phi) a.grad_phi[t * (N * N) + k] = s;
      } else if constexpr (FUSED) {
        if (k < N * N + N) {
          if (a.grad_alpha) a.grad_alpha[t * N + (k - N * N)] = s;
        } else {
          if (a.grad_beta) a.grad_beta[t * N + (k - N * N - N)] = s;
        }
      }
      if constexpr (PROJ) fin[threadIdx.y][k] = s;
    }
  }
  if constexpr (PROJ) {
    __syncthreads();
    // grad_v_j = rho_j - sum_i Phi_ij rho_i + beta-part_j
    // (reference ops/stream_mix_small_nb.py:379-384)
    if (tok_ok && a.grad_v != nullptr && threadIdx.x < N) {
      const int j = threadIdx.x;
      const float* fr = fin[threadIdx.y];
      float ptr = 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) ptr = fmaf(phi[i * N + j], fr[N * N + i], ptr);
      a.grad_v[t * N + j] = (fr[N * N + j] - ptr) + fr[N * N + N + j];
    }
  }
}

// ============================================================== geometry
struct MixGeometry {
  dim3 grid;
  dim3 block;
  int nchunk;
  int passes;
};

inline MixGeometry mix_geometry(int64_t T, int64_t D, int E) {
  MixGeometry g;
  const int64_t nchunk = (D + E - 1) / E;
  int64_t tx = ((nchunk + 31) / 32) * 32;
  if (tx > kMaxCtaThreads) tx = kMaxCtaThreads;
  if (tx < 32) tx = 32;
  g.nchunk = static_cast<int>(nchunk);
  g.passes = static_cast<int>((nchunk + tx - 1) / tx);
  int64_t ty = kMaxCtaThreads / tx;
  if (ty > T) ty = T;
  if (ty < 1) ty = 1;
  g.block = dim3(static_cast<unsigned>(tx), static_cast<unsigned>(ty), 1);
  g.grid = dim3(static_cast<unsigned>((T + ty - 1) / ty), 1, 1);
  return g;
}

// ============================================================== launchers
// Declared here, instantiated per stream dtype in mix_*.cu.
template <typename T, typename P, bool FUSED, bool PROJ, bool VECTOR>
int launch_mix_fwd(int n, const MixGeometry& g, const MixFwdArgs& a, cudaStream_t s) {
  switch (n) {
#define HC_CASE(NN)                                                                 \
  case NN:                                                                          \
    mix_fwd_kernel<T, P, NN, FUSED, PROJ, VECTOR><<<g.grid, g.block, 0, s>>>(a); \
    break;
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

template <typename T, typename P, bool FUSED, bool PROJ, bool VECTOR>
int launch_mix_bwd(int n, const MixGeometry& g, const MixBwdArgs& a, cudaStream_t s) {
  switch (n) {
#define HC_CASE(NN)                                                                 \
  case NN:                                                                          \
    mix_bwd_kernel<T, P, NN, FUSED, PROJ, VECTOR><<<g.grid, g.block, 0, s>>>(a); \
    break;
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

// Per-dtype entry points (defined in mix_f32.cu / mix_f16.cu / mix_bf16.cu).
// `param_is_f32` selects P = float, else P = T.
int mix_fwd_f32(bool fused, bool proj, bool vec, bool param_is_f32, int n, const MixGeometry& g,
                const MixFwdArgs& a, cudaStream_t s);
int mix_fwd_f16(bool fused, bool proj, bool vec, bool param_is_f32, int n, const MixGeometry& g,
                const MixFwdArgs& a, cudaStream_t s);
int mix_fwd_bf16(bool fused, bool proj, bool vec, bool param_is_f32, int n, const MixGeometry& g,
                 const MixFwdArgs& a, cudaStream_t s);
int mix_bwd_f32(bool fused, bool proj, bool vec, bool param_is_f32, int n, const MixGeometry& g,
                const MixBwdArgs& a, cudaStream_t s);
int mix_bwd_f16(bool fused, bool proj, bool vec, bool param_is_f32, int n, const MixGeometry& g,
                const MixBwdArgs& a, cudaStream_t s);
int mix_bwd_bf16(bool fused, bool proj, bool vec, bool param_is_f32, int n, const MixGeometry& g,
                 const MixBwdArgs& a, cudaStream_t s);

}  // namespace hc
