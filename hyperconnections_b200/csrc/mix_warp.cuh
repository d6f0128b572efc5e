// mix_warp.cuh — warp-autonomous, TMA-fed stream-mixing kernels (fast path).
//
// Every warp of a persistent CTA owns whole tokens (token gw, gw + stride,
// ...) and its own ring of shared-memory stages with one mbarrier each. Lane 0
// issues the bulk copies (cp.async.bulk, no multicast) of the warp's next
// token-slices; all lanes wait on the stage's barrier, compute, and after a
// __syncwarp lane 0 refills the stage. Warps never wait for one another: there
// is no CTA-wide barrier, so the SM always has independent warps to issue
// from, and the bytes in flight per SM are warps x stages x stage bytes.
//
// A stage holds one token-slice of every input row the kernel needs:
//   forward  fused: x (n rows), f (1)          add: x (n), Y (n)
//   backward fused: g_x (n), x (n), g_u (1), f (1)   add: g (n), x (n)
// laid out [tensor][row][pitch]. When a token fits one slice the rows of one
// tensor are contiguous in HBM and land with ONE bulk copy per tensor.
//
// Lane l of a warp reads W consecutive 32-bit words of every row at word
// offset seg*32*W + l*W (conflict-free shared-memory reads, coalesced global
// stores). Because a token stays on one warp, the backward's per-token sums
// (grad_Phi / grad_H, grad_alpha, grad_beta, the projection terms) accumulate
// in registers over all slices and fold with one warp transpose-reduce.
//
// Every wait is bounded (kWaitLimit polls); a warp that gives up counts it in
// a device counter (hc_wait_timeouts), drains its own copies with another
// bounded wait and stops.
#pragma once

#include <algorithm>
#include <cmath>

#include "mix_kernels.cuh"

namespace hc {

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 1-D bulk copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kWarpMaxStages = 8;
constexpr int kWarpMaxWarps = 16;

// Count of bounded waits that gave up (one counter per translation unit; read
// and cleared by hc_wait_timeouts()).
static __device__ unsigned int g_mix_wait_timeouts;

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ------------------------------------------------------------------ words
// 32-bit word <-> K elements in fp32.
template <typename T> struct Word;
template <> struct Word<float> {
  static constexpr int K = 1;
  __device__ static __forceinline__ void get(uint32_t w, float* f) { f[0] = __uint_as_float(w); }
  __device__ static __forceinline__ uint32_t put(const float* f) { return __float_as_uint(f[0]); }
};
template <> struct Word<__nv_bfloat16> {
  static constexpr int K = 2;
  __device__ static __forceinline__ void get(uint32_t w, float* f) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xffff0000u);
  }
  __device__ static __forceinline__ uint32_t put(const float* f) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[0], f[1]);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Word<__half> {
  static constexpr int K = 2;
  __device__ static __forceinline__ void get(uint32_t w, float* f) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 p = __half22float2(h);
    f[0] = p.x;
    f[1] = p.y;
  }
  __device__ static __forceinline__ uint32_t put(const float* f) {
    __half2 h = __floats2half2_rn(f[0], f[1]);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// W consecutive 32-bit words from shared memory / to global memory.
template <int W> struct Words {
  uint32_t w[W];
};
template <int W>
__device__ __forceinline__ Words<W> lds_words(const uint8_t* p) {
  Words<W> r;
  if constexpr (W == 4) {
    uint4 q = *reinterpret_cast<const uint4*>(p);
    r.w[0] = q.x; r.w[1] = q.y; r.w[2] = q.z; r.w[3] = q.w;
  } else if constexpr (W == 2) {
    uint2 q = *reinterpret_cast<const uint2*>(p);
    r.w[0] = q.x; r.w[1] = q.y;
  } else {
    r.w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
  return r;
}
template <int W>
__device__ __forceinline__ void stg_words(void* p, const uint32_t* w) {
  if constexpr (W == 4) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
  } else if constexpr (W == 2) {
    asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(w[0]), "r"(w[1]) : "memory");
  } else {
    asm volatile("st.global.u32 [%0], %1;" ::"l"(p), "r"(w[0]) : "memory");
  }
}

// ------------------------------------------------------------------ geometry
struct WarpGeometry {
  int warps;        // warps per CTA
  int stages;       // stages per warp
  int sl;           // elements per slice
  int ns;           // slices per token
  int pitch;        // shared-memory row pitch (elements)
  int stage_bytes;  // rows * pitch * element size
  int grid;         // CTAs
  int smem_bytes;   // dynamic shared memory per CTA
};

// Issue the bulk copies of one token-slice into a stage.
template <typename T, int NIN>
__device__ __forceinline__ void warp_issue(const WarpGeometry& geo, int64_t D, uint8_t* stage, uint64_t* bar,
                                           int64_t t, int p, const void* const* base, const int* rows) {
  constexpr int es = sizeof(T);
  const int64_t d0 = static_cast<int64_t>(p) * geo.sl;
  const int len = static_cast<int>(std::min<int64_t>(geo.sl, D - d0));
  int rtot = 0;
#pragma unroll
  for (int k = 0; k < NIN; ++k) rtot += rows[k];
  mbar_expect_tx(bar, static_cast<uint32_t>(rtot * len * es));
  uint8_t* dst = stage;
#pragma unroll
  for (int k = 0; k < NIN; ++k) {
    const T* src = static_cast<const T*>(base[k]) + t * rows[k] * D;
    if (geo.ns == 1) {
      bulk_g2s(dst, src, static_cast<uint32_t>(rows[k] * D * es), bar);
    } else {
      for (int r = 0; r < rows[k]; ++r)
        bulk_g2s(dst + static_cast<size_t>(r) * geo.pitch * es, src + r * D + d0, static_cast<uint32_t>(len * es),
                 bar);
    }
    dst += static_cast<size_t>(rows[k]) * geo.pitch * es;
  }
}

// Per-token parameters in registers.
template <typename P, int N, bool FUSED, bool PROJ>
struct TokParams {
  float phi[N * N];
  float vv[PROJ ? N : 1], cc[PROJ ? N : 1];
  float al[FUSED ? N : 1], be[FUSED ? N : 1];
  __device__ __forceinline__ void load(const void* phi_p, const void* v_p, const float* alpha, const float* beta,
                                       int64_t t) {
    load_params<P, N * N>(static_cast<const P*>(phi_p) + t * (N * N), phi);
    if constexpr (PROJ) {
      load_params<P, N>(static_cast<const P*>(v_p) + t * N, vv);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float pv = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) pv = fmaf(phi[i * N + j], vv[j], pv);
        cc[i] = vv[i] - pv;
      }
    }
    if constexpr (FUSED) {
      load_params<float, N>(alpha + t * N, al);
      load_params<float, N>(beta + t * N, be);
    }
  }
};

// ================================================================= forward
// Warps per CTA at most: 16 (128 registers per thread) for n <= 4, 8 above.
constexpr int warp_cap(int n) { return n <= 4 ? kWarpMaxWarps : kWarpMaxWarps / 2; }

template <typename T, typename P, int N, bool FUSED, bool PROJ, int W>
__global__ void __launch_bounds__(warp_cap(N) * 32, 1)
mix_fwd_warp_kernel(const MixFwdArgs a, const WarpGeometry geo) {
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int NS = FUSED ? 1 : N;  // rows of the second input
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;   // elements per warp access
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bars[kWarpMaxWarps][kWarpMaxStages];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* wsm = smem + static_cast<size_t>(warp) * geo.stages * geo.stage_bytes;
  uint64_t* full = bars[warp];
  if (lane == 0) {
    for (int s = 0; s < geo.stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int64_t T_ = a.T, D = a.D;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * geo.warps + warp;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * geo.warps;
  const int64_t ntok = gw < T_ ? (T_ - gw + stride - 1) / stride : 0;
  const int64_t nitems = ntok * geo.ns;
  const void* base[2] = {a.x, a.src};
  const int rows[2] = {N, NS};
  const size_t rowb = static_cast<size_t>(geo.pitch) * es;

  if (lane == 0)
    for (int64_t i = 0; i < nitems && i < geo.stages; ++i)
      warp_issue<T, 2>(geo, D, wsm + i * geo.stage_bytes, &full[i], gw + (i / geo.ns) * stride,
                       static_cast<int>(i % geo.ns), base, rows);

  TokParams<P, N, FUSED, PROJ> pr;
  int64_t i = 0;
  bool aborted = false;
  for (; i < nitems; ++i) {
    const int s = static_cast<int>(i % geo.stages);
    const int64_t t = gw + (i / geo.ns) * stride;
    const int p = static_cast<int>(i % geo.ns);
    if (p == 0) pr.load(a.phi, a.v, a.alpha, a.beta, t);
    if (!__all_sync(kFull, warp_wait(&full[s], static_cast<uint32_t>((i / geo.stages) & 1)))) {
      aborted = true;
      break;
    }
    const uint8_t* sb = wsm + static_cast<size_t>(s) * geo.stage_bytes;
    const int64_t d0 = static_cast<int64_t>(p) * geo.sl;
    const int len = static_cast<int>(std::min<int64_t>(geo.sl, D - d0));
    T* ot = static_cast<T*>(a.out) + t * N * D + d0;
    T* ut = FUSED ? static_cast<T*>(a.u) + t * D + d0 : nullptr;
    for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
      const uint8_t* q = sb + static_cast<size_t>(e0) * es;
      Words<W> xw[N], sw[NS];
#pragma unroll
      for (int j = 0; j < N; ++j) xw[j] = lds_words<W>(q + j * rowb);
#pragma unroll
      for (int i2 = 0; i2 < NS; ++i2) sw[i2] = lds_words<W>(q + (N + i2) * rowb);
      uint32_t ow[N][W], uw[W];
#pragma unroll
      for (int w = 0; w < W; ++w) {
        float xe[N][K], se[NS][K];
#pragma unroll
        for (int j = 0; j < N; ++j) Wd::get(xw[j].w[w], xe[j]);
#pragma unroll
        for (int i2 = 0; i2 < NS; ++i2) Wd::get(sw[i2].w[w], se[i2]);
        float av[K];
        if constexpr (PROJ) {
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < N; ++j) acc = fmaf(pr.vv[j], xe[j][e], acc);
            av[e] = acc;
          }
        }
        if constexpr (FUSED) {
          float uo[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < N; ++j) acc = fmaf(pr.al[j], xe[j][e], acc);
            uo[e] = acc;
          }
          uw[w] = Wd::put(uo);
        }
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) {
          float o[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < N; ++j) acc = fmaf(pr.phi[i2 * N + j], xe[j][e], acc);
            if constexpr (PROJ) acc = fmaf(pr.cc[i2], av[e], acc);
            if constexpr (FUSED) {
              acc = fmaf(pr.be[i2], se[0][e], acc);
            } else {
              acc = acc + se[i2][e];
            }
            o[e] = acc;
          }
          ow[i2][w] = Wd::put(o);
        }
      }
#pragma unroll
      for (int i2 = 0; i2 < N; ++i2) stg_words<W>(ot + i2 * D + e0, ow[i2]);
      if constexpr (FUSED) stg_words<W>(ut + e0, uw);
    }
    __syncwarp();
    if (lane == 0 && i + geo.stages < nitems) {
      fence_proxy_async_smem();
      const int64_t in = i + geo.stages;
      warp_issue<T, 2>(geo, D, wsm + static_cast<size_t>(s) * geo.stage_bytes, &full[s],
                       gw + (in / geo.ns) * stride, static_cast<int>(in % geo.ns), base, rows);
    }
  }
  if (aborted && lane == 0) {
    atomicAdd(&g_mix_wait_timeouts, 1u);
    for (int64_t j = i; j < nitems && j < i + geo.stages; ++j)  // drain this warp's copies
      warp_wait(&full[j % geo.stages], static_cast<uint32_t>((j / geo.stages) & 1));
  }
}

// ================================================================= backward
template <typename T, typename P, int N, bool FUSED, bool PROJ, int W>
__global__ void __launch_bounds__(warp_cap(N) * 32, 1)
mix_bwd_warp_kernel(const MixBwdArgs a, const WarpGeometry geo) {
  using Wd = Word<T>;
  using L = BwdLayout<N, FUSED, PROJ>;
  constexpr int K = Wd::K;
  constexpr int R = L::kR;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  constexpr int NIN = FUSED ? 4 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bars[kWarpMaxWarps][kWarpMaxStages];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* wsm = smem + static_cast<size_t>(warp) * geo.stages * geo.stage_bytes;
  uint64_t* full = bars[warp];
  if (lane == 0) {
    for (int s = 0; s < geo.stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int64_t T_ = a.T, D = a.D;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * geo.warps + warp;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * geo.warps;
  const int64_t ntok = gw < T_ ? (T_ - gw + stride - 1) / stride : 0;
  const int64_t nitems = ntok * geo.ns;
  const void* base[NIN];
  int rows[NIN];
  base[0] = a.g;
  base[1] = a.x;
  rows[0] = N;
  rows[1] = N;
  if constexpr (FUSED) {
    base[2] = a.gu;
    base[3] = a.f;
    rows[2] = 1;
    rows[3] = 1;
  }
  const size_t rowb = static_cast<size_t>(geo.pitch) * es;

  if (lane == 0)
    for (int64_t i = 0; i < nitems && i < geo.stages; ++i)
      warp_issue<T, NIN>(geo, D, wsm + i * geo.stage_bytes, &full[i], gw + (i / geo.ns) * stride,
                         static_cast<int>(i % geo.ns), base, rows);

  TokParams<P, N, FUSED, PROJ> pr;
  float acc[L::kPad];
  int64_t i = 0;
  bool aborted = false;
  for (; i < nitems; ++i) {
    const int s = static_cast<int>(i % geo.stages);
    const int64_t t = gw + (i / geo.ns) * stride;
    const int p = static_cast<int>(i % geo.ns);
    if (p == 0) {
      pr.load(a.phi, a.v, a.alpha, a.beta, t);
#pragma unroll
      for (int k = 0; k < L::kPad; ++k) acc[k] = 0.f;
    }
    if (!__all_sync(kFull, warp_wait(&full[s], static_cast<uint32_t>((i / geo.stages) & 1)))) {
      aborted = true;
      break;
    }
    const uint8_t* sb = wsm + static_cast<size_t>(s) * geo.stage_bytes;
    const int64_t d0 = static_cast<int64_t>(p) * geo.sl;
    const int len = static_cast<int>(std::min<int64_t>(geo.sl, D - d0));
    T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * N * D + d0 : nullptr;
    T* gft = (FUSED && a.grad_f) ? static_cast<T*>(a.grad_f) + t * D + d0 : nullptr;
    for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
      const uint8_t* q = sb + static_cast<size_t>(e0) * es;
      Words<W> gw_[N], xw[N], uw, fw;
#pragma unroll
      for (int r = 0; r < N; ++r) gw_[r] = lds_words<W>(q + r * rowb);
#pragma unroll
      for (int r = 0; r < N; ++r) xw[r] = lds_words<W>(q + (N + r) * rowb);
      if constexpr (FUSED) {
        uw = lds_words<W>(q + (2 * N) * rowb);
        fw = lds_words<W>(q + (2 * N + 1) * rowb);
      }
      uint32_t gxo[N][W], gfo[W];
#pragma unroll
      for (int w = 0; w < W; ++w) {
        float ge[N][K], xe[N][K], gue[K], fe[K];
#pragma unroll
        for (int r = 0; r < N; ++r) Wd::get(gw_[r].w[w], ge[r]);
#pragma unroll
        for (int r = 0; r < N; ++r) Wd::get(xw[r].w[w], xe[r]);
        if constexpr (FUSED) {
          Wd::get(uw.w[w], gue);
          Wd::get(fw.w[w], fe);
        }
        float av[K], bt[K];
        if constexpr (PROJ) {
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sa = 0.f, sb2 = 0.f;
#pragma unroll
            for (int j = 0; j < N; ++j) sa = fmaf(pr.vv[j], xe[j][e], sa);
#pragma unroll
            for (int i2 = 0; i2 < N; ++i2) sb2 = fmaf(ge[i2][e], pr.cc[i2], sb2);
            av[e] = sa;
            bt[e] = sb2;
          }
        }
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float o[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sacc = 0.f;
#pragma unroll
            for (int i2 = 0; i2 < N; ++i2) sacc = fmaf(pr.phi[i2 * N + j], ge[i2][e], sacc);
            if constexpr (PROJ) sacc = fmaf(pr.vv[j], bt[e], sacc);
            if constexpr (FUSED) sacc = fmaf(pr.al[j], gue[e], sacc);
            o[e] = sacc;
          }
          gxo[j][w] = Wd::put(o);
        }
        if constexpr (FUSED) {
          float o[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sacc = 0.f;
#pragma unroll
            for (int i2 = 0; i2 < N; ++i2) sacc = fmaf(pr.be[i2], ge[i2][e], sacc);
            o[e] = sacc;
          }
          gfo[w] = Wd::put(o);
        }
#pragma unroll
        for (int e = 0; e < K; ++e) {
#pragma unroll
          for (int j = 0; j < N; ++j) {
            float xv = xe[j][e];
            if constexpr (PROJ) xv = xv - pr.vv[j] * av[e];
#pragma unroll
            for (int i2 = 0; i2 < N; ++i2) acc[i2 * N + j] = fmaf(ge[i2][e], xv, acc[i2 * N + j]);
          }
          if constexpr (FUSED) {
#pragma unroll
            for (int j = 0; j < N; ++j) acc[N * N + j] = fmaf(gue[e], xe[j][e], acc[N * N + j]);
#pragma unroll
            for (int i2 = 0; i2 < N; ++i2) acc[N * N + N + i2] = fmaf(ge[i2][e], fe[e], acc[N * N + N + i2]);
          }
          if constexpr (PROJ) {
#pragma unroll
            for (int i2 = 0; i2 < N; ++i2) acc[N * N + i2] = fmaf(ge[i2][e], av[e], acc[N * N + i2]);
#pragma unroll
            for (int j = 0; j < N; ++j) acc[N * N + N + j] = fmaf(bt[e], xe[j][e], acc[N * N + N + j]);
          }
        }
      }
      if (gxt) {
#pragma unroll
        for (int j = 0; j < N; ++j) stg_words<W>(gxt + j * D + e0, gxo[j]);
      }
      if constexpr (FUSED) {
        if (gft) stg_words<W>(gft + e0, gfo);
      }
    }
    __syncwarp();
    if (lane == 0 && i + geo.stages < nitems) {
      fence_proxy_async_smem();
      const int64_t in = i + geo.stages;
      warp_issue<T, NIN>(geo, D, wsm + static_cast<size_t>(s) * geo.stage_bytes, &full[s],
                         gw + (in / geo.ns) * stride, static_cast<int>(in % geo.ns), base, rows);
    }
    if (p == geo.ns - 1) {
      // this warp's token is complete: fold the 32 lanes' partial sums
      float v[L::kPad];
#pragma unroll
      for (int k = 0; k < L::kPad; ++k) v[k] = acc[k];
      warp_transpose_reduce<R>(v, lane);  // lane l now holds sums [R*l, R*l + R)
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int k = lane * R + r;
        if (k < N * N) {
          if (a.grad_phi) a.grad_phi[t * (N * N) + k] = v[r];
        } else if (k < L::kAcc) {
          if constexpr (FUSED) {
            if (k < N * N + N) {
              if (a.grad_alpha) a.grad_alpha[t * N + (k - N * N)] = v[r];
            } else {
              if (a.grad_beta) a.grad_beta[t * N + (k - N * N - N)] = v[r];
            }
          }
        }
      }
      if constexpr (PROJ) {
        // grad_v_j = rho_j - sum_i Phi_ij rho_i + beta-part_j
        // (reference ops/stream_mix_small_nb.py:379-384)
        float rho[N], bp[N];
#pragma unroll
        for (int q2 = 0; q2 < N; ++q2) {
          rho[q2] = __shfl_sync(kFull, v[(N * N + q2) % R], (N * N + q2) / R);
          bp[q2] = __shfl_sync(kFull, v[(N * N + N + q2) % R], (N * N + N + q2) / R);
        }
        if (a.grad_v != nullptr && lane < N) {
          float out = 0.f;
#pragma unroll
          for (int j = 0; j < N; ++j) {
            if (j == lane) {
              float ptr = 0.f;
#pragma unroll
              for (int i2 = 0; i2 < N; ++i2) ptr = fmaf(pr.phi[i2 * N + j], rho[i2], ptr);
              out = (rho[j] - ptr) + bp[j];
            }
          }
          a.grad_v[t * N + lane] = out;
        }
      }
    }
  }
  if (aborted && lane == 0) {
    atomicAdd(&g_mix_wait_timeouts, 1u);
    for (int64_t j = i; j < nitems && j < i + geo.stages; ++j)
      warp_wait(&full[j % geo.stages], static_cast<uint32_t>((j / geo.stages) & 1));
  }
}

// ================================================================= host side
inline int warp_rows(bool bwd, bool fused, int n) {
  if (!bwd) return fused ? n + 1 : 2 * n;
  return fused ? 2 * n + 2 : 2 * n;
}

// Tuning knobs (0 = automatic), set through hc_set_mix_tuning().
struct WarpTuning {
  int stage_bytes;  // target bytes of one stage
  int stages;       // stages per warp
  int warps;        // warps per CTA
};
WarpTuning& warp_tuning();

// Geometry of the warp pipeline; false when the shape does not fit it.
// Requires D % (16 / esize) == 0 and 16-byte aligned stream bases.
inline bool warp_geometry(WarpGeometry& geo, bool bwd, bool fused, int n, int64_t T, int64_t D, int esize,
                          int num_sms) {
  if (T <= 0 || D <= 0 || D % (16 / esize) != 0) return false;
  const WarpTuning tune = warp_tuning();
  const int rows = warp_rows(bwd, fused, n);
  const int budget = 200 * 1024;
  const int wcap = warp_cap(n);
  int stages = tune.stages > 0 ? std::min(tune.stages, kWarpMaxStages) : 2;
  if (stages < 2) stages = 2;
  // slice: the whole token when its rows fit the stage target, else a
  // multiple of 64 elements
  const int64_t target =
      tune.stage_bytes > 0 ? tune.stage_bytes : std::max<int64_t>(2048, budget / (stages * wcap));
  int64_t sl = D;
  if (rows * D * esize > target) {
    sl = std::max<int64_t>(64, (target / (rows * esize)) / 64 * 64);
    if (sl >= D) sl = D;
  }
  geo.sl = static_cast<int>(sl);
  geo.ns = static_cast<int>((D + sl - 1) / sl);
  geo.pitch = geo.sl;
  geo.stage_bytes = static_cast<int>(rows * sl * esize);
  int wmax = budget / (stages * geo.stage_bytes);
  if (wmax > wcap) wmax = wcap;
  if (tune.warps > 0) wmax = std::min(wmax, tune.warps);
  if (wmax < 1) return false;
  // warps per CTA: among the last few counts that fit, the one whose last
  // round of tokens is fullest (tokens are dealt round-robin to warps)
  int best = wmax;
  double best_eff = 0.0;
  for (int w = wmax; w >= std::max(1, wmax - 4); --w) {
    const int64_t grid = std::min<int64_t>(num_sms, (T + w - 1) / w);
    const double per = static_cast<double>(T) / (grid * w);
    const double eff = per / std::ceil(per);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = w;
    }
  }
  geo.warps = best;
  geo.stages = stages;
  geo.smem_bytes = best * stages * geo.stage_bytes;
  geo.grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms, (T + best - 1) / best)));
  return true;
}

template <typename KernelT>
inline int warp_prepare(KernelT* kernel, int smem_bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
    return HC_ERR_LAUNCH;
  return HC_OK;
}

constexpr int kWarpW = 2;  // 32-bit words per lane access (8-byte accesses)

template <typename T, typename P, bool FUSED, bool PROJ>
int launch_mix_fwd_warp(int n, const WarpGeometry& geo, const MixFwdArgs& a, cudaStream_t s) {
  const dim3 block(geo.warps * 32, 1, 1);
  switch (n) {
#define HC_CASE(NN)                                                     \
  case NN: {                                                            \
    auto* k = mix_fwd_warp_kernel<T, P, NN, FUSED, PROJ, kWarpW>;       \
    if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;            \
    k<<<geo.grid, block, geo.smem_bytes, s>>>(a, geo);                  \
    break;                                                              \
  }
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

template <typename T, typename P, bool FUSED, bool PROJ>
int launch_mix_bwd_warp(int n, const WarpGeometry& geo, const MixBwdArgs& a, cudaStream_t s) {
  const dim3 block(geo.warps * 32, 1, 1);
  switch (n) {
#define HC_CASE(NN)                                                     \
  case NN: {                                                            \
    auto* k = mix_bwd_warp_kernel<T, P, NN, FUSED, PROJ, kWarpW>;       \
    if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;            \
    k<<<geo.grid, block, geo.smem_bytes, s>>>(a, geo);                  \
    break;                                                              \
  }
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

// Per-dtype entry points of the warp-pipelined kernels (mix_*.cu).
#define HC_DECLARE_WARP(SFX)                                                                                 \
  int mix_fwd_warp_##SFX(bool fused, bool proj, bool param_is_f32, int n, const WarpGeometry& g,             \
                         const MixFwdArgs& a, cudaStream_t s);                                               \
  int mix_bwd_warp_##SFX(bool fused, bool proj, bool param_is_f32, int n, const WarpGeometry& g,             \
                         const MixBwdArgs& a, cudaStream_t s);                                               \
  unsigned int mix_warp_take_timeouts_##SFX(bool reset);
HC_DECLARE_WARP(f32)
HC_DECLARE_WARP(f16)
HC_DECLARE_WARP(bf16)
#undef HC_DECLARE_WARP

}  // namespace hc
