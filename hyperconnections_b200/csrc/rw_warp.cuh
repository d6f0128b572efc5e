// rw_warp.cuh — width-read and mix + depth-write for a general backbone
// width m (1 <= m <= 4), forward and backward, on the shared-memory ring of
// mix_warp.cuh.
//
// Per token t (rows of D elements, fp32 arithmetic, I/O in the stream type):
//
//   read        u_k   = sum_j R_kj x_j                        k < m
//               (reference hyperconnections/cghc.py:410, ghc.py:116,
//                mhc.py:138, attnhc.py:154: einsum "b m n, b n d -> b m d")
//   mix-write   x'_i  = sum_j H_ij x_j [+ c_i (v^T x)] + sum_k W_ik f_k
//               with c = v - H v (the projected mix)
//               (reference cghc.py:417 write einsum "b n m, b m d -> b n d"
//                followed by stream_mix_add, cghc.py:449 ->
//                ops/stream_mix_small_nb.py:75-132, without materialising
//                the written term Y)
//
// Backward, given the upstream gradient g of the output rows:
//   read        grad_x_j = sum_k R_kj g_k           grad_R_kj = sum_d g_k x_j
//   mix-write   grad_x_j = sum_i H_ij g_i [+ v_j (c^T g)]
//               grad_f_k = sum_i W_ik g_i
//               grad_H_ij = sum_d g_i (x_j - v_j v^T x)   grad_W_ik = sum_d g_i f_k
//               grad_v as in stream_mix_small_nb.py:379-384
//
// The producer lane, the ring protocol and the geometry are those of the
// fused kernels (mix_warp.cuh); only the consumer arithmetic differs. Each
// per-token parameter row is fp32 ([T,m,n] R, [T,n,n] H, [T,n,m] W, [T,n] v).
#pragma once

#include "mix_warp.cuh"

namespace hc {

struct RwArgs {
  const void* x;    // [T,N,D]
  const void* f;    // [T,M,D]   mix-write input
  const void* g;    // upstream gradient: [T,M,D] (read) | [T,N,D] (mix-write)
  const float* R;   // [T,M,N]   read weights
  const float* H;   // [T,N,N]   transition matrices
  const float* W;   // [T,N,M]   write weights
  const float* v;   // [T,N]     projection direction (nullable)
  void* out;        // forward output: u [T,M,D] | x' [T,N,D]
  void* grad_x;     // [T,N,D]   nullable
  void* grad_f;     // [T,M,D]   nullable
  float* grad_R;    // [T,M,N]   nullable
  float* grad_H;    // [T,N,N]   nullable
  float* grad_W;    // [T,N,M]   nullable
  float* grad_v;    // [T,N]     nullable
  int64_t T;
  int64_t D;
};

// Warps per CTA and 32-bit words per lane access, from the register need:
// rows held per element and, in the backward, the per-token accumulators.
constexpr int rw_fwd_rows(int n, int m, bool mixw) { return mixw ? n + m : n; }
constexpr int rw_bwd_rows(int n, int m, bool mixw) { return mixw ? 2 * n + m : n + m; }
constexpr int rw_acc(int n, int m, bool mixw, bool proj) {
  return mixw ? n * n + n * m + (proj ? 2 * n : 0) : m * n;
}
constexpr int rw_fwd_cap(int n, int m, bool mixw) { return rw_fwd_rows(n, m, mixw) <= 6 ? 16 : 8; }
constexpr int rw_fwd_words(int n, int m, bool mixw) { return rw_fwd_rows(n, m, mixw) <= 6 ? 4 : 2; }
constexpr int rw_bwd_cap(int n, int m, bool mixw, bool proj) { return rw_acc(n, m, mixw, proj) <= 24 ? 12 : 8; }
constexpr int rw_bwd_words(int n, int m, bool mixw, bool proj) { return rw_acc(n, m, mixw, proj) <= 48 ? 2 : 1; }

template <int N, int M, bool MIXW, bool PROJ>
struct RwParams {
  static constexpr int KA = MIXW ? N * N : M * N;
  float a[KA];                     // R (read) or H (mix-write)
  float w[MIXW ? N * M : 1];       // W
  float vv[PROJ ? N : 1], cc[PROJ ? N : 1];
  __device__ __forceinline__ void load(const RwArgs& p, int64_t t) {
    if constexpr (MIXW) {
      load_params_keep<float, N * N>(p.H + t * (N * N), a);
      load_params_keep<float, N * M>(p.W + t * (N * M), w);
      if constexpr (PROJ) {
        load_params_keep<float, N>(p.v + t * N, vv);
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float hv = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) hv = fmaf(a[i * N + j], vv[j], hv);
          cc[i] = vv[i] - hv;
        }
      }
    } else {
      load_params_keep<float, M * N>(p.R + t * (M * N), a);
    }
  }
};

// ------------------------------------------------------------------ forward
// xsb / fsb: shared-memory rows of this token's slice (row pitch `pitch`).
template <typename T, int N, int M, bool MIXW, bool PROJ, int W>
__device__ __forceinline__ void rw_fwd_slice(const RwArgs& a, const RwParams<N, M, MIXW, PROJ>& pr,
                                             const uint8_t* xsb, const uint8_t* fsb, int pitch, int64_t t,
                                             int64_t d0, int len, int lane) {
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  constexpr int NO = MIXW ? N : M;  // output rows
  constexpr int NF = MIXW ? M : 1;
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* ot = static_cast<T*>(a.out) + t * NO * D + d0;
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> xw[N], fw[NF];
#pragma unroll
    for (int j = 0; j < N; ++j) xw[j] = lds_words<W>(xsb + eo + j * rowb);
    if constexpr (MIXW) {
#pragma unroll
      for (int k = 0; k < M; ++k) fw[k] = lds_words<W>(fsb + eo + k * rowb);
    }
    uint32_t ow[NO][W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      float xe[N][K], fe[NF][K];
#pragma unroll
      for (int j = 0; j < N; ++j) Wd::get(xw[j].w[w], xe[j]);
      if constexpr (MIXW) {
#pragma unroll
        for (int k = 0; k < M; ++k) Wd::get(fw[k].w[w], fe[k]);
      }
      float sv[K];
      if constexpr (PROJ) {
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) s = fmaf(pr.vv[j], xe[j][e], s);
          sv[e] = s;
        }
      }
#pragma unroll
      for (int i = 0; i < NO; ++i) {
        float o[K];
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) s = fmaf(pr.a[i * N + j], xe[j][e], s);
          if constexpr (MIXW) {
            if constexpr (PROJ) s = fmaf(pr.cc[i], sv[e], s);
#pragma unroll
            for (int k = 0; k < M; ++k) s = fmaf(pr.w[i * M + k], fe[k][e], s);
          }
          o[e] = s;
        }
        ow[i][w] = Wd::put(o);
      }
    }
#pragma unroll
    for (int i = 0; i < NO; ++i) stg_words<W>(ot + i * D + e0, ow[i]);
  }
}

template <typename T, int N, int M, bool MIXW, bool PROJ>
__global__ void __launch_bounds__(rw_fwd_cap(N, M, MIXW) * 32, 1)
rw_fwd_warp_kernel(const RwArgs a, const WarpGeometry geo) {
  constexpr int W = rw_fwd_words(N, M, MIXW);
  constexpr int es = sizeof(T);
  constexpr int NIN = MIXW ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ RingState st;
  pdl_launch_dependents();
  ring_init(st, geo.stages);
  pdl_wait_prior_grid();

  const int64_t T_ = a.T, D = a.D;
  const UnitMap um = unit_map(T_, geo.tpi);
  const int nunits = um.nunits;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = geo.stages, C = geo.consumers, ns = geo.ns;
  const uint32_t rowb = static_cast<uint32_t>(geo.pitch) * es;
  const uint32_t xregion = static_cast<uint32_t>(geo.tpi) * N * rowb;  // x rows of all tokens of a stage

  if (warp == 0) {
    if (lane < geo.producers) {
      const void* base[2] = {a.x, a.f};
      const int rows[2] = {N, M};
      ring_produce<T, NIN>(st, geo, smem, D, um, base, rows, lane);
    }
  } else if (warp - 1 < C) {
    const int c = warp - 1;
    RwParams<N, M, MIXW, PROJ> pr;
    RingCursor cur{c, 0u, c};
    for (int g0 = 0; g0 < nunits; g0 += C) {
      const int Wg = min(C, nunits - g0);
      if (c >= Wg) break;
      const int u = g0 + c;
      const int cnt = um.cnt(u, geo.tpi);
      const int64_t t0 = um.tok(u);
      pr.load(a, t0);  // overlaps the wait for the data
      bool ok = true;
      for (int p = 0; p < ns; ++p) {
        if (__any_sync(kFull, st.abort) || !ring_wait_item(st, cur, geo.wait_limit)) {
          if (lane == 0 && !st.abort) {
            report_timeout(&g_mix_wait_timeouts, geo.status);
            st.abort = 1;
          }
          ok = false;
          break;
        }
        const uint8_t* sb = smem + static_cast<size_t>(cur.s) * geo.stage_bytes;
        const int64_t d0 = static_cast<int64_t>(p) * geo.sl;
        const int len = static_cast<int>(std::min<int64_t>(geo.sl, D - d0));
        for (int tt = 0; tt < cnt; ++tt) {
          if (tt > 0) pr.load(a, t0 + tt);
          rw_fwd_slice<T, N, M, MIXW, PROJ, W>(a, pr, sb + tt * N * rowb, sb + xregion + tt * M * rowb,
                                               geo.pitch, t0 + tt, d0, len, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&st.empty[cur.s]);
        cur.advance(p + 1 < ns ? Wg : C, S);
      }
      if (!ok) break;
    }
  }
  ring_drain(st, S);
}

// ----------------------------------------------------------------- backward
// Accumulator slots per lane (summed over the lane's elements):
//   read       [0, M*N)                grad_R(k,j)
//   mix-write  [0, N*N)                grad_H(i,j)
//              [N*N, N*N+N*M)          grad_W(i,k)
//              PROJ: next N            rho_i = sum g_i (v^T x)
//                    next N            bp_j  = sum (c^T g) x_j
template <int N, int M, bool MIXW, bool PROJ>
struct RwLayout {
  static constexpr int kAcc = rw_acc(N, M, MIXW, PROJ);
  static constexpr int kR = (kAcc + 31) / 32;
  static constexpr int kPad = 32 * kR;
};

// gsb, xsb, fsb: shared-memory rows of the upstream gradient, x and f.
template <typename T, int N, int M, bool MIXW, bool PROJ, int W>
__device__ __forceinline__ void rw_bwd_slice(const RwArgs& a, const RwParams<N, M, MIXW, PROJ>& pr, float* acc,
                                             const uint8_t* gsb, const uint8_t* xsb, const uint8_t* fsb,
                                             int pitch, int64_t t, int64_t d0, int len, int lane) {
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  constexpr int NG = MIXW ? N : M;  // upstream-gradient rows
  constexpr int NF = MIXW ? M : 1;
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * N * D + d0 : nullptr;
  T* gft = (MIXW && a.grad_f) ? static_cast<T*>(a.grad_f) + t * M * D + d0 : nullptr;
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> gw[NG], xw[N], fw[NF];
#pragma unroll
    for (int r = 0; r < NG; ++r) gw[r] = lds_words<W>(gsb + eo + r * rowb);
#pragma unroll
    for (int r = 0; r < N; ++r) xw[r] = lds_words<W>(xsb + eo + r * rowb);
    if constexpr (MIXW) {
#pragma unroll
      for (int r = 0; r < M; ++r) fw[r] = lds_words<W>(fsb + eo + r * rowb);
    }
    uint32_t gxo[N][W], gfo[NF][W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      float ge[NG][K], xe[N][K], fe[NF][K];
#pragma unroll
      for (int r = 0; r < NG; ++r) Wd::get(gw[r].w[w], ge[r]);
#pragma unroll
      for (int r = 0; r < N; ++r) Wd::get(xw[r].w[w], xe[r]);
      if constexpr (MIXW) {
#pragma unroll
        for (int r = 0; r < M; ++r) Wd::get(fw[r].w[w], fe[r]);
      }
      float sv[K], bt[K];  // v^T x and c^T g per element (projection)
      if constexpr (PROJ) {
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f, b = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) s = fmaf(pr.vv[j], xe[j][e], s);
#pragma unroll
          for (int i = 0; i < N; ++i) b = fmaf(ge[i][e], pr.cc[i], b);
          sv[e] = s;
          bt[e] = b;
        }
      }
      // grad_x_j = sum_r A_rj g_r (A = R or H) [+ v_j c^T g]
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float o[K];
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int r = 0; r < NG; ++r) s = fmaf(pr.a[r * N + j], ge[r][e], s);
          if constexpr (PROJ) s = fmaf(pr.vv[j], bt[e], s);
          o[e] = s;
        }
        gxo[j][w] = Wd::put(o);
      }
      if constexpr (MIXW) {
#pragma unroll
        for (int k = 0; k < M; ++k) {
          float o[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < N; ++i) s = fmaf(pr.w[i * M + k], ge[i][e], s);
            o[e] = s;
          }
          gfo[k][w] = Wd::put(o);
        }
      }
      // parameter-gradient partial sums
#pragma unroll
      for (int e = 0; e < K; ++e) {
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float xv = xe[j][e];
          if constexpr (PROJ) xv = xv - pr.vv[j] * sv[e];
#pragma unroll
          for (int r = 0; r < NG; ++r) acc[r * N + j] = fmaf(ge[r][e], xv, acc[r * N + j]);
        }
        if constexpr (MIXW) {
#pragma unroll
          for (int i = 0; i < N; ++i) {
#pragma unroll
            for (int k = 0; k < M; ++k) acc[N * N + i * M + k] = fmaf(ge[i][e], fe[k][e], acc[N * N + i * M + k]);
          }
          if constexpr (PROJ) {
            constexpr int o0 = N * N + N * M;
#pragma unroll
            for (int i = 0; i < N; ++i) acc[o0 + i] = fmaf(ge[i][e], sv[e], acc[o0 + i]);
#pragma unroll
            for (int j = 0; j < N; ++j) acc[o0 + N + j] = fmaf(bt[e], xe[j][e], acc[o0 + N + j]);
          }
        }
      }
    }
    if (gxt) {
#pragma unroll
      for (int j = 0; j < N; ++j) stg_words<W>(gxt + j * D + e0, gxo[j]);
    }
    if constexpr (MIXW) {
      if (gft) {
#pragma unroll
        for (int k = 0; k < M; ++k) stg_words<W>(gft + k * D + e0, gfo[k]);
      }
    }
  }
}

// Fold the 32 lanes' partial sums of one token and write its parameter
// gradients.
template <int N, int M, bool MIXW, bool PROJ>
__device__ __forceinline__ void rw_bwd_finish(const RwArgs& a, const RwParams<N, M, MIXW, PROJ>& pr,
                                              const float* acc, int64_t t, int lane) {
  using L = RwLayout<N, M, MIXW, PROJ>;
  constexpr int R = L::kR;
  float v[L::kPad];
#pragma unroll
  for (int k = 0; k < L::kPad; ++k) v[k] = acc[k];
  warp_transpose_reduce<R>(v, lane);  // lane l now holds sums [R*l, R*l + R)
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int k = lane * R + r;
    if constexpr (!MIXW) {
      if (k < M * N && a.grad_R) a.grad_R[t * (M * N) + k] = v[r];
    } else {
      if (k < N * N) {
        if (a.grad_H) a.grad_H[t * (N * N) + k] = v[r];
      } else if (k < N * N + N * M) {
        if (a.grad_W) a.grad_W[t * (N * M) + (k - N * N)] = v[r];
      }
    }
  }
  if constexpr (MIXW && PROJ) {
    // grad_v_j = rho_j - sum_i H_ij rho_i + bp_j
    constexpr int o0 = N * N + N * M;
    float rho[N], bp[N];
#pragma unroll
    for (int q = 0; q < N; ++q) {
      rho[q] = __shfl_sync(kFull, v[(o0 + q) % R], (o0 + q) / R);
      bp[q] = __shfl_sync(kFull, v[(o0 + N + q) % R], (o0 + N + q) / R);
    }
    if (a.grad_v != nullptr && lane < N) {
      float out = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        if (j == lane) {
          float ht = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) ht = fmaf(pr.a[i * N + j], rho[i], ht);
          out = (rho[j] - ht) + bp[j];
        }
      }
      a.grad_v[t * N + lane] = out;
    }
  }
}

// ------------------------------------ mix-write backward, Gram on the tensor cores
// Half-precision streams cut into slices at n >= 5: the consumer computes
// grad_x and grad_f of each slice on the CUDA cores (rw_bwd_grads_slice, no
// sums) and the token's Gram M = G [X; F]^T (N x (N + M), g rows against the
// x and f rows) on the tensor cores (gram_mma_slice, ring rows padded by 16
// bytes); every parameter gradient then follows from M (rw_gram_finish):
//   grad_H_ij = M_ij [- v_j rho_i],  grad_W_ik = M_i,N+k,
//   rho_i = sum_d g_i v^T x = sum_j v_j M_ij,  bp_j = sum_d (c^T g) x_j = sum_i c_i M_ij,
//   grad_v_j = rho_j - sum_i H_ij rho_i + bp_j (ops/stream_mix_small_nb.py:379-384).
constexpr bool rw_gram_mma(int n, bool mixw, int esize) { return mixw && n >= 5 && gram_mma_dtype(esize); }
// 8 warps (7 consumers, the count sliced backward rings run): H, W, v and c
// stay in registers (up to 112 floats at n = 8, m = 4), 255 registers a thread.
constexpr int kRwMmaWarps = 8;

// Geometry of the tensor-core mix-write backward (rw_gram_mma, slices):
// swizzled TMA stages for even n and D a multiple of 64 (regions g, x of n
// rows and f of m rows; an odd number of 128-byte lines a row, 9 stages of a
// kGramBudget ring), else the plain slices in 16-byte padded rows. `plain` is
// the ring geometry of the shape (rows 2n + m, slices).
inline bool rw_mma_geometry(WarpGeometry& geo, const WarpGeometry& plain, int n, int m, int64_t T, int64_t D,
                            int esize, bool allow_swizzle) {
  if (allow_swizzle && n % 2 == 0 && D % kTmaChunk == 0 && T * n < (int64_t(1) << 31)) {
    const auto stage_of = [&](int nc) {
      return 2 * swz_region_bytes(n, nc * kTmaChunk, esize) + swz_region_bytes(m, nc * kTmaChunk, esize);
    };
    const int64_t chunks = D / kTmaChunk;
    int nc_max = 1;
    for (int c = 3; c <= 255 && stage_of(c) <= kGramBudget / 9; c += 2) nc_max = c;
    const int64_t ns = (chunks + nc_max - 1) / nc_max;
    const int nc = static_cast<int>((chunks + ns - 1) / ns) | 1;
    geo = plain;
    geo.sl = nc * kTmaChunk;
    geo.pitch = geo.sl;
    geo.ns = static_cast<int>((D + geo.sl - 1) / geo.sl);
    geo.stage_bytes = stage_of(nc);
    geo.gram_mma = kGramSwizzled;
    if (geo.ns > 1 && ring_stage(geo, kRwMmaWarps, T, sm_count(), kSwzAlign, kGramBudget)) return true;
  }
  geo = plain;
  geo.pitch = geo.sl + kGramPad;
  geo.stage_bytes = (2 * n + m) * geo.pitch * esize;
  geo.gram_mma = kGramPadded;
  if (ring_stage(geo, kRwMmaWarps, T, sm_count())) return true;
  geo = plain;
  return false;
}

// SWZ: the stage's g region is swizzled (nc lines a row); otherwise row-major
// with `pitch` elements per row.
template <typename T, int N, int M, bool PROJ, int W, bool SWZ = false>
__device__ __forceinline__ void rw_bwd_grads_slice(const RwArgs& a, const RwParams<N, M, true, PROJ>& pr,
                                                   const uint8_t* gsb, int pitch, int64_t t, int64_t d0, int len,
                                                   int lane, int nc = 0) {
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * N * D + d0 : nullptr;
  T* gft = a.grad_f ? static_cast<T*>(a.grad_f) + t * M * D + d0 : nullptr;
  if (gxt == nullptr && gft == nullptr) return;
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> gw[N];
#pragma unroll
    for (int r = 0; r < N; ++r)
      gw[r] = lds_words<W>(stage_at<SWZ>(gsb, rowb, nc, r, static_cast<int>(eo)));
    uint32_t gxo[N][W], gfo[M][W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      float ge[N][K];
#pragma unroll
      for (int r = 0; r < N; ++r) Wd::get(gw[r].w[w], ge[r]);
      float bt[K];  // c^T g per element (projection)
      if constexpr (PROJ) {
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float b = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) b = fmaf(ge[i][e], pr.cc[i], b);
          bt[e] = b;
        }
      }
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float o[K];
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int r = 0; r < N; ++r) s = fmaf(pr.a[r * N + j], ge[r][e], s);
          if constexpr (PROJ) s = fmaf(pr.vv[j], bt[e], s);
          o[e] = s;
        }
        gxo[j][w] = Wd::put(o);
      }
#pragma unroll
      for (int k = 0; k < M; ++k) {
        float o[K];
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) s = fmaf(pr.w[i * M + k], ge[i][e], s);
          o[e] = s;
        }
        gfo[k][w] = Wd::put(o);
      }
    }
    if (gxt) {
#pragma unroll
      for (int j = 0; j < N; ++j) stg_words<W>(gxt + j * D + e0, gxo[j]);
    }
    if (gft) {
#pragma unroll
      for (int k = 0; k < M; ++k) stg_words<W>(gft + k * D + e0, gfo[k]);
    }
  }
}

// The token's parameter gradients from its Gram M (row-major N x (N + M) in
// shared memory); lane i < N handles row i of grad_H and grad_W and entry i of
// grad_v. Register arrays are indexed with constants only.
template <int N, int M, bool PROJ>
__device__ __forceinline__ void rw_gram_finish(const RwArgs& a, const RwParams<N, M, true, PROJ>& pr,
                                               const float* gram, int64_t t, int lane) {
  constexpr int C = N + M;
  const int i = lane < N ? lane : 0;
  const float* row = gram + i * C;
  float rho = 0.f, bp = 0.f;
  if constexpr (PROJ) {
#pragma unroll
    for (int j = 0; j < N; ++j) rho = fmaf(pr.vv[j], row[j], rho);
#pragma unroll
    for (int q = 0; q < N; ++q) bp = fmaf(pr.cc[q], gram[q * C + i], bp);  // column i
  }
  float rho_all[PROJ ? N : 1];
  if constexpr (PROJ) {
#pragma unroll
    for (int q = 0; q < N; ++q) rho_all[q] = __shfl_sync(kFull, rho, q);
  }
  if (lane < N) {
    if (a.grad_H) {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float h = row[j];
        if constexpr (PROJ) h = fmaf(-pr.vv[j], rho, h);
        a.grad_H[t * (N * N) + i * N + j] = h;
      }
    }
    if (a.grad_W) {
#pragma unroll
      for (int k = 0; k < M; ++k) a.grad_W[t * (N * M) + i * M + k] = row[N + k];
    }
    if constexpr (PROJ) {
      if (a.grad_v) {
        float ht = 0.f;  // sum_q H_q,i rho_q, column i of H with a constant index
#pragma unroll
        for (int j = 0; j < N; ++j) {
          if (j == i) {
#pragma unroll
            for (int q = 0; q < N; ++q) ht = fmaf(pr.a[q * N + j], rho_all[q], ht);
          }
        }
        a.grad_v[t * N + i] = (rho - ht) + bp;
      }
    }
  }
  __syncwarp();
}

// Side rows of the mix-write backward (geo.side): the m rows of f of a
// token (contiguous in HBM) are copied by the consumer warp into one of two
// slots of its own with 16-byte cp.async while it computes the previous
// token, instead of riding in the ring as a small bulk copy (see side_fetch,
// mix_warp.cuh). The ring then carries the 2n rows of g and x.
template <typename T, int M>
__device__ __forceinline__ void rw_side_fetch(uint8_t* slot, const RwArgs& a, int64_t t, int lane) {
  const int64_t bytes = static_cast<int64_t>(M) * a.D * static_cast<int64_t>(sizeof(T));
  const int chunks = static_cast<int>(bytes / 16);
  const uint8_t* f = static_cast<const uint8_t*>(a.f) + t * bytes;
  for (int i = lane; i < chunks; i += 32)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(slot + i * 16)), "l"(f + i * 16)
                 : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <typename T, int N, int M, bool MIXW, bool PROJ, bool MMA = false, bool SWZ = false>
__global__ void __launch_bounds__((MMA ? kRwMmaWarps : rw_bwd_cap(N, M, MIXW, PROJ)) * 32, 1)
rw_bwd_warp_kernel(const RwArgs a, const WarpGeometry geo, const __grid_constant__ RingMaps maps) {
  static_assert(!MMA || (MIXW && sizeof(T) == 2), "the tensor-core Gram is a mix-write, half-precision path");
  static_assert(!SWZ || MMA, "swizzled stages belong to the tensor-core Gram");
  using L = RwLayout<N, M, MIXW, PROJ>;
  constexpr int W = MMA ? 2 : rw_bwd_words(N, M, MIXW, PROJ);
  constexpr int NT = (N + M + 7) / 8;
  __shared__ float gram_all[MMA ? (kWarpMaxWarps - 1) * N * (N + M) : 1];
  constexpr int es = sizeof(T);
  constexpr int NG = MIXW ? N : M;
  constexpr int NIN = MIXW ? 3 : 2;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // swizzled stages start on a 1024-byte boundary (kSwzAlign bytes of slack)
  uint8_t* const smem = SWZ ? smem_raw + ((kSwzAlign - (smem_u32(smem_raw) & (kSwzAlign - 1))) & (kSwzAlign - 1))
                            : smem_raw;
  __shared__ RingState st;
  pdl_launch_dependents();
  ring_init(st, geo.stages);
  pdl_wait_prior_grid();

  const int64_t T_ = a.T, D = a.D;
  const UnitMap um = unit_map(T_, geo.tpi);
  const int nunits = um.nunits;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = geo.stages, C = geo.consumers, ns = geo.ns;
  const uint32_t rowb = static_cast<uint32_t>(geo.pitch) * es;
  const uint32_t greg = static_cast<uint32_t>(geo.tpi) * NG * rowb;  // g rows of all tokens of a stage
  const uint32_t xreg = static_cast<uint32_t>(geo.tpi) * N * rowb;   // x rows of all tokens of a stage

  if (warp == 0) {
    if (lane < geo.producers) {
      const void* base[3] = {a.g, a.x, a.f};
      const int rows[3] = {NG, N, M};
      if (MIXW && geo.side) {
        ring_produce<T, 2>(st, geo, smem, D, um, base, rows, lane, &maps);
      } else {
        ring_produce<T, NIN>(st, geo, smem, D, um, base, rows, lane, &maps);
      }
    }
  } else if (warp - 1 < C) {
    const int c = warp - 1;
    RwParams<N, M, MIXW, PROJ> pr;
    float acc[MMA ? 1 : L::kPad];
    float cg[MMA ? NT : 1][4];  // tensor-core Gram accumulators of the token
    float* gram = gram_all + (MMA ? c * N * (N + M) : 0);
    // side rows (geo.side: mix-write, whole tokens one an item, no
    // tensor-core Gram): two slots of this consumer after the ring's stages
    constexpr bool SIDE_OK = MIXW && !MMA;
    const bool side = SIDE_OK && geo.side;
    const size_t side_slot_bytes = static_cast<size_t>(M) * D * es;
    uint8_t* const side_base =
        smem + static_cast<size_t>(S) * geo.stage_bytes + static_cast<size_t>(c) * 2 * side_slot_bytes;
    int side_slot = 0;
    const uint8_t* side_cur = nullptr;  // the current token's slot
    if constexpr (SIDE_OK) {
      if (side && c < nunits) rw_side_fetch<T, M>(side_base, a, um.tok(c), lane);
    }
    RingCursor cur{c, 0u, c};
    for (int g0 = 0; g0 < nunits; g0 += C) {
      const int Wg = min(C, nunits - g0);
      if (c >= Wg) break;
      const int u = g0 + c;
      const int cnt = um.cnt(u, geo.tpi);
      const int64_t t0 = um.tok(u);
      pr.load(a, t0);  // overlaps the wait for the data
      bool ok = true;
      for (int p = 0; p < ns; ++p) {
        if (__any_sync(kFull, st.abort) || !ring_wait_item(st, cur, geo.wait_limit)) {
          if (lane == 0 && !st.abort) {
            report_timeout(&g_mix_wait_timeouts, geo.status);
            st.abort = 1;
          }
          ok = false;
          break;
        }
        const uint8_t* sb = smem + static_cast<size_t>(cur.s) * geo.stage_bytes;
        const int64_t d0 = static_cast<int64_t>(p) * geo.sl;
        const int len = static_cast<int>(std::min<int64_t>(geo.sl, D - d0));
        if constexpr (SIDE_OK) {
          if (side) {  // this token's f rows landed in its slot; start the next token's
            side_cur = side_base + side_slot * side_slot_bytes;
            if (u + C < nunits) {
              rw_side_fetch<T, M>(side_base + (side_slot ^ 1) * side_slot_bytes, a, um.tok(u + C), lane);
              asm volatile("cp.async.wait_group 1;" ::: "memory");
            } else {
              asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            __syncwarp();
            side_slot ^= 1;
          }
        }
        for (int tt = 0; tt < cnt; ++tt) {
          const int64_t t = t0 + tt;
          if (p == 0) {
            if (tt > 0) pr.load(a, t);
            if constexpr (MMA) {
#pragma unroll
              for (int k = 0; k < NT; ++k) cg[k][0] = cg[k][1] = cg[k][2] = cg[k][3] = 0.f;
            } else {
#pragma unroll
              for (int k = 0; k < L::kPad; ++k) acc[k] = 0.f;
            }
          }
          const uint8_t* gs = sb + tt * NG * rowb;
          const uint8_t* xs = sb + greg + tt * N * rowb;
          const uint8_t* fs = sb + greg + xreg + tt * M * rowb;
          if constexpr (SIDE_OK) {
            if (side) fs = side_cur;  // tpi == 1
          }
          if constexpr (SWZ) {  // swizzled regions g, x, f (tpi == 1)
            xs = sb + swz_region_bytes(N, geo.sl, es);
            fs = xs + swz_region_bytes(N, geo.sl, es);
          }
          if constexpr (MMA) {
            const int nc = geo.sl / kTmaChunk;
            rw_bwd_grads_slice<T, N, M, PROJ, W, SWZ>(a, pr, gs, geo.pitch, t, d0, len, lane, nc);
            gram_mma_slice<T, N, 0, N, M, SWZ>(cg, gs, nullptr, xs, fs, reinterpret_cast<const uint8_t*>(st.zrow),
                                               rowb, nc, len, lane);
            if (p == ns - 1) {  // token complete
              gram_mma_store<N, N + M>(gram, cg, lane);
              rw_gram_finish<N, M, PROJ>(a, pr, gram, t, lane);
            }
          } else {
            rw_bwd_slice<T, N, M, MIXW, PROJ, W>(a, pr, acc, gs, xs, fs, geo.pitch, t, d0, len, lane);
            if (p == ns - 1) rw_bwd_finish<N, M, MIXW, PROJ>(a, pr, acc, t, lane);  // token complete
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&st.empty[cur.s]);
        cur.advance(p + 1 < ns ? Wg : C, S);
      }
      if (!ok) break;
    }
    if constexpr (SIDE_OK) {
      if (side) asm volatile("cp.async.wait_all;" ::: "memory");  // no copy lands after the CTA is gone
    }
  }
  ring_drain(st, S);
}

// ------------------------------------------------------- generic fallback
// Any D and any element alignment (the ring needs D % (16 / esize) == 0 and
// 16-byte aligned rows), any 1 <= m <= 4 <= n <= 8 combination: one warp per
// token, lanes over the elements, runtime n and m. Used for small or odd
// block sizes, where the token is a few hundred bytes at most.
constexpr int kRwGenericWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kRwGenericWarps * 32)
rw_fwd_generic_kernel(const RwArgs a, int n, int m, bool mixw) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kRwGenericWarps + (threadIdx.x >> 5);
  if (t >= a.T) return;
  const int64_t D = a.D;
  const bool proj = mixw && a.v != nullptr;
  float A[64], Wm[32], vv[8], cc[8];
  const int ka = mixw ? n * n : m * n;
  const float* ap = mixw ? a.H + t * n * n : a.R + t * m * n;
  for (int k = 0; k < ka; ++k) A[k] = ap[k];
  if (mixw) {
    for (int k = 0; k < n * m; ++k) Wm[k] = a.W[t * n * m + k];
    if (proj) {
      for (int i = 0; i < n; ++i) vv[i] = a.v[t * n + i];
      for (int i = 0; i < n; ++i) {
        float hv = 0.f;
        for (int j = 0; j < n; ++j) hv = fmaf(A[i * n + j], vv[j], hv);
        cc[i] = vv[i] - hv;
      }
    }
  }
  const T* xt = static_cast<const T*>(a.x) + t * n * D;
  const T* ft = mixw ? static_cast<const T*>(a.f) + t * m * D : nullptr;
  const int no = mixw ? n : m;
  T* ot = static_cast<T*>(a.out) + t * no * D;
  for (int64_t d = lane; d < D; d += 32) {
    float xe[8], fe[4];
    for (int j = 0; j < n; ++j) xe[j] = Elem<T>::to_f(xt[j * D + d]);
    if (mixw) {
      for (int k = 0; k < m; ++k) fe[k] = Elem<T>::to_f(ft[k * D + d]);
    }
    float s = 0.f;
    if (proj) {
      for (int j = 0; j < n; ++j) s = fmaf(vv[j], xe[j], s);
    }
    for (int i = 0; i < no; ++i) {
      float o = 0.f;
      for (int j = 0; j < n; ++j) o = fmaf(A[i * n + j], xe[j], o);
      if (mixw) {
        if (proj) o = fmaf(cc[i], s, o);
        for (int k = 0; k < m; ++k) o = fmaf(Wm[i * m + k], fe[k], o);
      }
      ot[i * D + d] = Elem<T>::from_f(o);
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kRwGenericWarps * 32)
rw_bwd_generic_kernel(const RwArgs a, int n, int m, bool mixw) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kRwGenericWarps + (threadIdx.x >> 5);
  if (t >= a.T) return;
  const int64_t D = a.D;
  const bool proj = mixw && a.v != nullptr;
  const int ng = mixw ? n : m;
  float A[64], Wm[32], vv[8], cc[8];
  const int ka = mixw ? n * n : m * n;
  const float* ap = mixw ? a.H + t * n * n : a.R + t * m * n;
  for (int k = 0; k < ka; ++k) A[k] = ap[k];
  if (mixw) {
    for (int k = 0; k < n * m; ++k) Wm[k] = a.W[t * n * m + k];
    if (proj) {
      for (int i = 0; i < n; ++i) vv[i] = a.v[t * n + i];
      for (int i = 0; i < n; ++i) {
        float hv = 0.f;
        for (int j = 0; j < n; ++j) hv = fmaf(A[i * n + j], vv[j], hv);
        cc[i] = vv[i] - hv;
      }
    }
  }
  // slots: [0, ka) grad_A; [64, 64 + n*m) grad_W; [96, 96 + n) rho; [104, 104 + n) bp
  float acc[112];
  for (int k = 0; k < 112; ++k) acc[k] = 0.f;
  const T* gt = static_cast<const T*>(a.g) + t * ng * D;
  const T* xt = static_cast<const T*>(a.x) + t * n * D;
  const T* ft = mixw ? static_cast<const T*>(a.f) + t * m * D : nullptr;
  T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * n * D : nullptr;
  T* gft = (mixw && a.grad_f) ? static_cast<T*>(a.grad_f) + t * m * D : nullptr;
  for (int64_t d = lane; d < D; d += 32) {
    float ge[8], xe[8], fe[4];
    for (int r = 0; r < ng; ++r) ge[r] = Elem<T>::to_f(gt[r * D + d]);
    for (int j = 0; j < n; ++j) xe[j] = Elem<T>::to_f(xt[j * D + d]);
    if (mixw) {
      for (int k = 0; k < m; ++k) fe[k] = Elem<T>::to_f(ft[k * D + d]);
    }
    float s = 0.f, b = 0.f;
    if (proj) {
      for (int j = 0; j < n; ++j) s = fmaf(vv[j], xe[j], s);
      for (int i = 0; i < n; ++i) b = fmaf(ge[i], cc[i], b);
    }
    for (int j = 0; j < n; ++j) {
      float o = 0.f;
      for (int r = 0; r < ng; ++r) o = fmaf(A[r * n + j], ge[r], o);
      if (proj) o = fmaf(vv[j], b, o);
      if (gxt) gxt[j * D + d] = Elem<T>::from_f(o);
    }
    if (mixw) {
      for (int k = 0; k < m; ++k) {
        float o = 0.f;
        for (int i = 0; i < n; ++i) o = fmaf(Wm[i * m + k], ge[i], o);
        if (gft) gft[k * D + d] = Elem<T>::from_f(o);
      }
    }
    for (int j = 0; j < n; ++j) {
      const float xv = proj ? xe[j] - vv[j] * s : xe[j];
      for (int r = 0; r < ng; ++r) acc[r * n + j] = fmaf(ge[r], xv, acc[r * n + j]);
    }
    if (mixw) {
      for (int i = 0; i < n; ++i)
        for (int k = 0; k < m; ++k) acc[64 + i * m + k] = fmaf(ge[i], fe[k], acc[64 + i * m + k]);
      if (proj) {
        for (int i = 0; i < n; ++i) acc[96 + i] = fmaf(ge[i], s, acc[96 + i]);
        for (int j = 0; j < n; ++j) acc[104 + j] = fmaf(b, xe[j], acc[104 + j]);
      }
    }
  }
  for (int k = 0; k < ka; ++k) {
    const float sum = warp_sum(acc[k]);
    float* dst = mixw ? a.grad_H : a.grad_R;
    if (lane == 0 && dst) dst[t * ka + k] = sum;
  }
  if (mixw) {
    for (int k = 0; k < n * m; ++k) {
      const float sum = warp_sum(acc[64 + k]);
      if (lane == 0 && a.grad_W) a.grad_W[t * n * m + k] = sum;
    }
    if (proj) {
      float rho[8], bp[8];
      for (int i = 0; i < n; ++i) rho[i] = warp_sum(acc[96 + i]);
      for (int j = 0; j < n; ++j) bp[j] = warp_sum(acc[104 + j]);
      if (lane == 0 && a.grad_v) {
        for (int j = 0; j < n; ++j) {
          float ht = 0.f;
          for (int i = 0; i < n; ++i) ht = fmaf(A[i * n + j], rho[i], ht);
          a.grad_v[t * n + j] = (rho[j] - ht) + bp[j];
        }
      }
    }
  }
}

// ------------------------------------------------------------- launchers
// Supported (n, m) for the ring kernels: 1 <= m <= min(n, 4), n <= 8.
inline bool rw_ring_supported(int n, int m) { return n >= 1 && n <= 8 && m >= 1 && m <= 4 && m <= n; }

template <typename T, bool BWD, bool MIXW, bool PROJ, int N, int M>
int rw_launch_one(const WarpGeometry& geo_in, const RwArgs& a, cudaStream_t s) {
  WarpGeometry geo = geo_in;
  geo.status = timeout_word(s);
  const dim3 block((geo.consumers + 1) * 32, 1, 1);
  if constexpr (BWD) {
    RingMaps maps{};
    if constexpr (rw_gram_mma(N, MIXW, sizeof(T))) {
      if constexpr (N % 2 == 0) {
        if (geo.gram_mma == kGramSwizzled) {
          const void* base[3] = {a.g, a.x, a.f};
          const int rows[3] = {N, N, M};
          if (ring_tensor_maps_swz(geo, maps, base, rows, 3, a.T, a.D, sizeof(T))) {
            geo.tma = 1;
            auto* k = rw_bwd_warp_kernel<T, N, M, MIXW, PROJ, true, true>;
            if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;
            return launch_ring(k, geo.grid, (geo.consumers + 1) * 32, geo.smem_bytes, s, a, geo, maps);
          }
          // no swizzled maps: the padded rows
          WarpGeometry plain = geo;
          if (!ring_geometry(plain, rw_bwd_rows(N, M, MIXW), kRwMmaWarps, a.T, a.D, sizeof(T), sm_count(), true) ||
              !rw_mma_geometry(geo, plain, N, M, a.T, a.D, sizeof(T), false))
            return HC_ERR_LAUNCH;
          geo.status = timeout_word(s);
          prefer_bwd_consumers(geo, 4);
          prefer_producers(geo);
        }
      }
      if (geo.gram_mma == kGramPadded) {
        auto* k = rw_bwd_warp_kernel<T, N, M, MIXW, PROJ, true>;
        if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;
        return launch_ring(k, geo.grid, (geo.consumers + 1) * 32, geo.smem_bytes, s, a, geo, maps);
      }
    }
    if (geo.gram_mma) return HC_ERR_LAUNCH;  // not reached: the geometry sets it only for this path
    auto* k = rw_bwd_warp_kernel<T, N, M, MIXW, PROJ>;
    if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;
    return launch_ring(k, geo.grid, block, geo.smem_bytes, s, a, geo, maps);
  } else {
    auto* k = rw_fwd_warp_kernel<T, N, M, MIXW, PROJ>;
    if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;
    return launch_ring(k, geo.grid, block, geo.smem_bytes, s, a, geo);
  }
}

template <typename T, bool BWD, bool MIXW, bool PROJ, int N>
int rw_launch_m(int m, const WarpGeometry& geo, const RwArgs& a, cudaStream_t s) {
  switch (m) {
    case 1: return rw_launch_one<T, BWD, MIXW, PROJ, N, 1>(geo, a, s);
    case 2: if constexpr (N >= 2) return rw_launch_one<T, BWD, MIXW, PROJ, N, 2>(geo, a, s); break;
    case 3: if constexpr (N >= 3) return rw_launch_one<T, BWD, MIXW, PROJ, N, 3>(geo, a, s); break;
    case 4: if constexpr (N >= 4) return rw_launch_one<T, BWD, MIXW, PROJ, N, 4>(geo, a, s); break;
    default: break;
  }
  return HC_ERR_UNSUPPORTED_N;
}

template <typename T, bool BWD, bool MIXW, bool PROJ>
int rw_launch_ring(int n, int m, const WarpGeometry& geo, const RwArgs& a, cudaStream_t s) {
  switch (n) {
    case 1: return rw_launch_m<T, BWD, MIXW, PROJ, 1>(m, geo, a, s);
    case 2: return rw_launch_m<T, BWD, MIXW, PROJ, 2>(m, geo, a, s);
    case 3: return rw_launch_m<T, BWD, MIXW, PROJ, 3>(m, geo, a, s);
    case 4: return rw_launch_m<T, BWD, MIXW, PROJ, 4>(m, geo, a, s);
    case 5: return rw_launch_m<T, BWD, MIXW, PROJ, 5>(m, geo, a, s);
    case 6: return rw_launch_m<T, BWD, MIXW, PROJ, 6>(m, geo, a, s);
    case 7: return rw_launch_m<T, BWD, MIXW, PROJ, 7>(m, geo, a, s);
    case 8: return rw_launch_m<T, BWD, MIXW, PROJ, 8>(m, geo, a, s);
    default: return HC_ERR_UNSUPPORTED_N;
  }
}

// Register caps of the (n, m, mode) the launcher picked (host side mirror of
// the kernels' __launch_bounds__).
inline int rw_cap(bool bwd, int n, int m, bool mixw, bool proj) {
  return bwd ? rw_bwd_cap(n, m, mixw, proj) : rw_fwd_cap(n, m, mixw);
}
inline int rw_rows(bool bwd, int n, int m, bool mixw) { return bwd ? rw_bwd_rows(n, m, mixw) : rw_fwd_rows(n, m, mixw); }

template <typename T>
int rw_launch_generic(bool bwd, int n, int m, bool mixw, const RwArgs& a, cudaStream_t s) {
  const int64_t blocks = (a.T + kRwGenericWarps - 1) / kRwGenericWarps;
  if (bwd) {
    rw_bwd_generic_kernel<T><<<static_cast<unsigned>(blocks), kRwGenericWarps * 32, 0, s>>>(a, n, m, mixw);
  } else {
    rw_fwd_generic_kernel<T><<<static_cast<unsigned>(blocks), kRwGenericWarps * 32, 0, s>>>(a, n, m, mixw);
  }
  return launch_status();
}

// Per-dtype, per-direction entry points (rw_<dtype>_<dir>.cu).
#define HC_DECLARE_RW(SFX)                                                                                  \
  int rw_fwd_##SFX(bool ring, bool mixw, bool proj, int n, int m, const WarpGeometry& g, const RwArgs& a,   \
                   cudaStream_t s);                                                                         \
  int rw_bwd_##SFX(bool ring, bool mixw, bool proj, int n, int m, const WarpGeometry& g, const RwArgs& a,   \
                   cudaStream_t s);                                                                         \
  unsigned int rw_fwd_take_timeouts_##SFX(bool reset);                                                      \
  unsigned int rw_bwd_take_timeouts_##SFX(bool reset);
HC_DECLARE_RW(f32)
HC_DECLARE_RW(f16)
HC_DECLARE_RW(bf16)
#undef HC_DECLARE_RW

}  // namespace hc
