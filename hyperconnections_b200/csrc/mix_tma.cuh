// mix_tma.cuh — persistent, TMA-fed stream-mixing kernels (the fast path).
//
// HBM -> shared memory moves with the bulk-copy engine (cp.async.bulk,
// completion counted on an mbarrier), so the bytes in flight per SM are set
// by the pipeline depth (STAGES x stage bytes, up to ~200 KB) rather than by
// how many threads can hold loads in registers. One CTA per SM walks its share
// of "tiles"; a tile is TOK consecutive tokens x one D-slice of DS elements,
// and holds every input row the kernel needs for those tokens and columns:
//
//   forward  fused: x (n rows), f (1 row)        add: x (n rows), Y (n rows)
//   backward fused: g_x (n), x (n), g_u (1), f (1)  add: g (n), x (n)
//
// Inside a stage the rows of one input tensor are stored [token][row][pitch]
// (pitch = D when a token fits one slice, so a whole tile of that tensor is
// ONE contiguous bulk copy; otherwise one copy per row slice). Thread (ty, tx)
// of the CTA handles token ty of the tile and the 16-byte chunk tx of the
// slice across all rows: shared-memory reads are 16-byte, conflict-free, and
// outputs leave with 16-byte st.global from registers. Slices of one token
// group run back-to-back on the same CTA, so the backward's per-token
// reductions accumulate in registers across slices and are folded (warp
// transpose-reduce + shared memory) after the last slice — no atomics, no
// global scratch.
//
// Synchronisation: one mbarrier per stage ("full"); thread 0 issues a stage's
// copies with arrive.expect_tx and refills the stage after the CTA-wide
// barrier that ends its use. Every wait is bounded: after kWaitLimit polls the
// kernel counts a timeout (read by hc_wait_timeouts), drains its own copies
// with another bounded wait, and returns.
#pragma once

#include <algorithm>

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
constexpr int kTmaMaxThreads = 512;  // per CTA: 128 registers per thread at one CTA per SM

// Count of bounded waits that gave up (one counter per translation unit;
// read and cleared by hc_wait_timeouts()).
static __device__ unsigned int g_mix_wait_timeouts;

// ------------------------------------------------------------------ words
// A 16-byte chunk is 4 32-bit words; a word holds K = 4 / sizeof(T) elements.
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

// ------------------------------------------------------------------ args
struct TmaGeometry {
  int tok;          // tokens per tile
  int tx;           // threads per token (multiple of 32)
  int ns;           // D-slices per token
  int ds;           // elements per slice (= tx * chunk elements)
  int pitch;        // shared-memory row pitch in elements
  int stages;       // pipeline depth
  int stage_bytes;  // bytes of one stage
  int64_t ngroups;  // ceil(T / tok)
  int grid;         // CTAs (persistent)
  int smem_bytes;   // dynamic shared memory per CTA
};

struct TmaState {
  uint64_t full[16];
  int abort;
};

// Issues the copies of sequence item j (group g, slice p) into stage s.
// NIN tensors; rows[k] rows per token; base[k] their global bases.
template <typename T, int NIN>
__device__ __forceinline__ void tma_issue(const TmaGeometry& geo, int64_t T_, int64_t D, uint8_t* stage,
                                          uint64_t* bar, int64_t g, int p, const void* const* base,
                                          const int* rows) {
  constexpr int es = sizeof(T);
  const int64_t t0 = g * geo.tok;
  const int cnt = static_cast<int>(min(static_cast<int64_t>(geo.tok), T_ - t0));
  const int64_t d0 = static_cast<int64_t>(p) * geo.ds;
  const int len = static_cast<int>(min(static_cast<int64_t>(geo.ds), D - d0));
  int rtot = 0;
#pragma unroll
  for (int k = 0; k < NIN; ++k) rtot += rows[k];
  mbar_expect_tx(bar, static_cast<uint32_t>(cnt) * rtot * len * es);
  uint8_t* dst = stage;
#pragma unroll
  for (int k = 0; k < NIN; ++k) {
    const T* src = static_cast<const T*>(base[k]);
    if (geo.ns == 1) {  // whole tokens: one contiguous copy per tensor
      bulk_g2s(dst, src + t0 * rows[k] * D, static_cast<uint32_t>(cnt * rows[k] * D * es), bar);
    } else {
      for (int tk = 0; tk < cnt; ++tk)
        for (int r = 0; r < rows[k]; ++r)
          bulk_g2s(dst + (static_cast<size_t>(tk) * rows[k] + r) * geo.pitch * es,
                   src + ((t0 + tk) * rows[k] + r) * D + d0, static_cast<uint32_t>(len * es), bar);
    }
    dst += static_cast<size_t>(geo.tok) * rows[k] * geo.pitch * es;
  }
}

// Bounded wait on a stage barrier; on timeout counts it and flags the CTA.
__device__ __forceinline__ bool tma_wait(uint64_t* bar, uint32_t parity, int* abort_flag) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicAdd(&g_mix_wait_timeouts, 1u);
  *abort_flag = 1;
  return false;
}

// After an abort: wait (bounded) for every stage that may still have copies
// in flight, so that none lands in shared memory after the CTA exits.
__device__ __forceinline__ void tma_drain(TmaState& st, const TmaGeometry& geo, int64_t j_next,
                                          int64_t j_end) {
  if (threadIdx.x != 0 || threadIdx.y != 0) return;
  for (int64_t j = j_next; j < j_end && j < j_next + geo.stages; ++j) {
    const int s = static_cast<int>(j % geo.stages);
    const uint32_t par = static_cast<uint32_t>((j / geo.stages) & 1);
    for (uint32_t i = 0; i < kWaitLimit; ++i)
      if (mbar_try_wait(&st.full[s], par)) break;
  }
}

// ================================================================= forward
template <typename T, typename P, int N, bool FUSED, bool PROJ>
__global__ void __launch_bounds__(kTmaMaxThreads, 1)
mix_fwd_tma_kernel(const MixFwdArgs a, const TmaGeometry geo) {
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int E = 4 * K;  // elements per 16-byte chunk
  constexpr int NS = FUSED ? 1 : N;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ TmaState st;

  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < geo.stages; ++s) mbar_init(&st.full[s], 1);
    st.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t T_ = a.T, D = a.D;
  const void* const base[2] = {a.x, a.src};
  const int rows[2] = {N, NS};
  // sequence item j -> (group, slice) for this CTA
  const int64_t my_groups = (geo.ngroups - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const int64_t jend = blockIdx.x < geo.ngroups ? my_groups * geo.ns : 0;
  auto group_of = [&](int64_t j) { return blockIdx.x + (j / geo.ns) * gridDim.x; };

  if (tid == 0)
    for (int64_t j = 0; j < jend && j < geo.stages; ++j)
      tma_issue<T, 2>(geo, T_, D, smem + static_cast<size_t>(j) * geo.stage_bytes, &st.full[j], group_of(j),
                      static_cast<int>(j % geo.ns), base, rows);

  const size_t xreg = static_cast<size_t>(geo.tok) * N * geo.pitch * sizeof(T);
  float phi[N * N], vv[N], cc[N], al[N], be[N];
  int64_t cur_group = -1;

  int64_t j = 0;
  for (; j < jend; ++j) {
    const int s = static_cast<int>(j % geo.stages);
    const int64_t g = group_of(j);
    const int p = static_cast<int>(j % geo.ns);
    const int64_t t = g * geo.tok + threadIdx.y;
    const bool tok_ok = t < T_;
    if (g != cur_group) {  // parameters of this thread's token
      cur_group = g;
      const int64_t ts = tok_ok ? t : 0;
      load_params<P, N * N>(static_cast<const P*>(a.phi) + ts * (N * N), phi);
      if constexpr (PROJ) {
        load_params<P, N>(static_cast<const P*>(a.v) + ts * N, vv);
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float pv = 0.f;
#pragma unroll
          for (int jj = 0; jj < N; ++jj) pv = fmaf(phi[i * N + jj], vv[jj], pv);
          cc[i] = vv[i] - pv;
        }
      }
      if constexpr (FUSED) {
        load_params<float, N>(a.alpha + ts * N, al);
        load_params<float, N>(a.beta + ts * N, be);
      }
    }
    tma_wait(&st.full[s], static_cast<uint32_t>((j / geo.stages) & 1), &st.abort);
    const int64_t d_el = static_cast<int64_t>(p) * geo.ds + static_cast<int64_t>(threadIdx.x) * E;
    if (tok_ok && d_el < D && !st.abort) {
      const uint8_t* sb = smem + static_cast<size_t>(s) * geo.stage_bytes;
      const uint32_t* xs = reinterpret_cast<const uint32_t*>(
          sb + (static_cast<size_t>(threadIdx.y) * N * geo.pitch + threadIdx.x * E) * sizeof(T));
      const uint32_t* ss = reinterpret_cast<const uint32_t*>(
          sb + xreg + (static_cast<size_t>(threadIdx.y) * NS * geo.pitch + threadIdx.x * E) * sizeof(T));
      const size_t rstride = static_cast<size_t>(geo.pitch) * sizeof(T) / 4;  // words per row
      uint4 xq[N], sq[NS];
#pragma unroll
      for (int jj = 0; jj < N; ++jj) xq[jj] = *reinterpret_cast<const uint4*>(xs + jj * rstride);
#pragma unroll
      for (int i = 0; i < NS; ++i) sq[i] = *reinterpret_cast<const uint4*>(ss + i * rstride);
      uint32_t ow[N][4], uw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        float xe[N][K], se[NS][K];
#pragma unroll
        for (int jj = 0; jj < N; ++jj) Wd::get((&xq[jj].x)[w], xe[jj]);
#pragma unroll
        for (int i = 0; i < NS; ++i) Wd::get((&sq[i].x)[w], se[i]);
        float av[K];
        if constexpr (PROJ) {
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sacc = 0.f;
#pragma unroll
            for (int jj = 0; jj < N; ++jj) sacc = fmaf(vv[jj], xe[jj][e], sacc);
            av[e] = sacc;
          }
        }
        if constexpr (FUSED) {
          float uo[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sacc = 0.f;
#pragma unroll
            for (int jj = 0; jj < N; ++jj) sacc = fmaf(al[jj], xe[jj][e], sacc);
            uo[e] = sacc;
          }
          uw[w] = Wd::put(uo);
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float o[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sacc = 0.f;
#pragma unroll
            for (int jj = 0; jj < N; ++jj) sacc = fmaf(phi[i * N + jj], xe[jj][e], sacc);
            if constexpr (PROJ) sacc = fmaf(cc[i], av[e], sacc);
            if constexpr (FUSED) {
              sacc = fmaf(be[i], se[0][e], sacc);
            } else {
              sacc = sacc + se[i][e];
            }
            o[e] = sacc;
          }
          ow[i][w] = Wd::put(o);
        }
      }
      T* ot = static_cast<T*>(a.out) + t * N * D + d_el;
#pragma unroll
      for (int i = 0; i < N; ++i) st_v4(ot + i * D, make_uint4(ow[i][0], ow[i][1], ow[i][2], ow[i][3]));
      if constexpr (FUSED) st_v4(static_cast<T*>(a.u) + t * D + d_el, make_uint4(uw[0], uw[1], uw[2], uw[3]));
    }
    __syncthreads();  // stage s fully consumed by every thread
    if (st.abort) break;
    if (tid == 0 && j + geo.stages < jend) {
      fence_proxy_async_smem();
      const int64_t jn = j + geo.stages;
      tma_issue<T, 2>(geo, T_, D, smem + static_cast<size_t>(s) * geo.stage_bytes, &st.full[s], group_of(jn),
                      static_cast<int>(jn % geo.ns), base, rows);
    }
  }
  if (st.abort) tma_drain(st, geo, j, jend);
}

// ================================================================= backward
template <typename T, typename P, int N, bool FUSED, bool PROJ>
__global__ void __launch_bounds__(kTmaMaxThreads, 1)
mix_bwd_tma_kernel(const MixBwdArgs a, const TmaGeometry geo) {
  using Wd = Word<T>;
  using L = BwdLayout<N, FUSED, PROJ>;
  constexpr int K = Wd::K;
  constexpr int E = 4 * K;
  constexpr int R = L::kR;
  constexpr int NIN = FUSED ? 4 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ TmaState st;
  __shared__ float red[kTmaMaxThreads / 32][L::kPad];  // one row per warp
  __shared__ float fin[PROJ ? kTmaMaxThreads / 32 : 1][PROJ ? L::kAcc : 1];

  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < geo.stages; ++s) mbar_init(&st.full[s], 1);
    st.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t T_ = a.T, D = a.D;
  const void* base[NIN];
  base[0] = a.g;
  base[1] = a.x;
  if constexpr (FUSED) {
    base[2] = a.gu;
    base[3] = a.f;
  }
  int rows[NIN];
  rows[0] = N;
  rows[1] = N;
  if constexpr (FUSED) {
    rows[2] = 1;
    rows[3] = 1;
  }
  const int64_t my_groups = (geo.ngroups - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const int64_t jend = blockIdx.x < geo.ngroups ? my_groups * geo.ns : 0;
  auto group_of = [&](int64_t j) { return blockIdx.x + (j / geo.ns) * gridDim.x; };

  if (tid == 0)
    for (int64_t j = 0; j < jend && j < geo.stages; ++j)
      tma_issue<T, NIN>(geo, T_, D, smem + static_cast<size_t>(j) * geo.stage_bytes, &st.full[j], group_of(j),
                        static_cast<int>(j % geo.ns), base, rows);

  const size_t rowbytes = static_cast<size_t>(geo.pitch) * sizeof(T);
  const size_t greg = static_cast<size_t>(geo.tok) * N * rowbytes;  // size of the g (and x) region
  const size_t ureg = static_cast<size_t>(geo.tok) * rowbytes;      // size of the g_u (and f) region
  const size_t rstride = rowbytes / 4;

  float phi[N * N], vv[N], cc[N], al[N], be[N];
  float acc[L::kPad];
  const int lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int wid = threadIdx.y * nw + (threadIdx.x >> 5);

  int64_t j = 0;
  for (; j < jend; ++j) {
    const int s = static_cast<int>(j % geo.stages);
    const int64_t g = group_of(j);
    const int p = static_cast<int>(j % geo.ns);
    const int64_t t = g * geo.tok + threadIdx.y;
    const bool tok_ok = t < T_;
    if (p == 0) {
      const int64_t ts = tok_ok ? t : 0;
      load_params<P, N * N>(static_cast<const P*>(a.phi) + ts * (N * N), phi);
      if constexpr (PROJ) {
        load_params<P, N>(static_cast<const P*>(a.v) + ts * N, vv);
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float pv = 0.f;
#pragma unroll
          for (int jj = 0; jj < N; ++jj) pv = fmaf(phi[i * N + jj], vv[jj], pv);
          cc[i] = vv[i] - pv;
        }
      }
      if constexpr (FUSED) {
        load_params<float, N>(a.alpha + ts * N, al);
        load_params<float, N>(a.beta + ts * N, be);
      }
#pragma unroll
      for (int k = 0; k < L::kPad; ++k) acc[k] = 0.f;
    }
    tma_wait(&st.full[s], static_cast<uint32_t>((j / geo.stages) & 1), &st.abort);
    const int64_t d_el = static_cast<int64_t>(p) * geo.ds + static_cast<int64_t>(threadIdx.x) * E;
    if (tok_ok && d_el < D && !st.abort) {
      const uint8_t* sb = smem + static_cast<size_t>(s) * geo.stage_bytes;
      const size_t coff = static_cast<size_t>(threadIdx.x) * E * sizeof(T);
      const uint32_t* gs = reinterpret_cast<const uint32_t*>(sb + threadIdx.y * N * rowbytes + coff);
      const uint32_t* xs = reinterpret_cast<const uint32_t*>(sb + greg + threadIdx.y * N * rowbytes + coff);
      uint4 gq[N], xq[N], uq, fq;
#pragma unroll
      for (int i = 0; i < N; ++i) gq[i] = *reinterpret_cast<const uint4*>(gs + i * rstride);
#pragma unroll
      for (int i = 0; i < N; ++i) xq[i] = *reinterpret_cast<const uint4*>(xs + i * rstride);
      if constexpr (FUSED) {
        uq = *reinterpret_cast<const uint4*>(sb + 2 * greg + threadIdx.y * rowbytes + coff);
        fq = *reinterpret_cast<const uint4*>(sb + 2 * greg + ureg + threadIdx.y * rowbytes + coff);
      }
      uint32_t gxw[N][4], gfw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        float ge[N][K], xe[N][K], gue[K], fe[K];
#pragma unroll
        for (int i = 0; i < N; ++i) Wd::get((&gq[i].x)[w], ge[i]);
#pragma unroll
        for (int i = 0; i < N; ++i) Wd::get((&xq[i].x)[w], xe[i]);
        if constexpr (FUSED) {
          Wd::get((&uq.x)[w], gue);
          Wd::get((&fq.x)[w], fe);
        }
        float av[K], bt[K];
        if constexpr (PROJ) {
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sa = 0.f, sb2 = 0.f;
#pragma unroll
            for (int jj = 0; jj < N; ++jj) sa = fmaf(vv[jj], xe[jj][e], sa);
#pragma unroll
            for (int i = 0; i < N; ++i) sb2 = fmaf(ge[i][e], cc[i], sb2);
            av[e] = sa;
            bt[e] = sb2;
          }
        }
#pragma unroll
        for (int jj = 0; jj < N; ++jj) {
          float o[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sacc = 0.f;
#pragma unroll
            for (int i = 0; i < N; ++i) sacc = fmaf(phi[i * N + jj], ge[i][e], sacc);
            if constexpr (PROJ) sacc = fmaf(vv[jj], bt[e], sacc);
            if constexpr (FUSED) sacc = fmaf(al[jj], gue[e], sacc);
            o[e] = sacc;
          }
          gxw[jj][w] = Wd::put(o);
        }
        if constexpr (FUSED) {
          float o[K];
#pragma unroll
          for (int e = 0; e < K; ++e) {
            float sacc = 0.f;
#pragma unroll
            for (int i = 0; i < N; ++i) sacc = fmaf(be[i], ge[i][e], sacc);
            o[e] = sacc;
          }
          gfw[w] = Wd::put(o);
        }
#pragma unroll
        for (int e = 0; e < K; ++e) {
#pragma unroll
          for (int jj = 0; jj < N; ++jj) {
            float xv = xe[jj][e];
            if constexpr (PROJ) xv = xv - vv[jj] * av[e];
#pragma unroll
            for (int i = 0; i < N; ++i) acc[i * N + jj] = fmaf(ge[i][e], xv, acc[i * N + jj]);
          }
          if constexpr (FUSED) {
#pragma unroll
            for (int jj = 0; jj < N; ++jj) acc[N * N + jj] = fmaf(gue[e], xe[jj][e], acc[N * N + jj]);
#pragma unroll
            for (int i = 0; i < N; ++i) acc[N * N + N + i] = fmaf(ge[i][e], fe[e], acc[N * N + N + i]);
          }
          if constexpr (PROJ) {
#pragma unroll
            for (int i = 0; i < N; ++i) acc[N * N + i] = fmaf(ge[i][e], av[e], acc[N * N + i]);
#pragma unroll
            for (int jj = 0; jj < N; ++jj) acc[N * N + N + jj] = fmaf(bt[e], xe[jj][e], acc[N * N + N + jj]);
          }
        }
      }
      if (a.grad_x) {
        T* gx = static_cast<T*>(a.grad_x) + t * N * D + d_el;
#pragma unroll
        for (int jj = 0; jj < N; ++jj)
          st_v4(gx + jj * D, make_uint4(gxw[jj][0], gxw[jj][1], gxw[jj][2], gxw[jj][3]));
      }
      if constexpr (FUSED) {
        if (a.grad_f) st_v4(static_cast<T*>(a.grad_f) + t * D + d_el, make_uint4(gfw[0], gfw[1], gfw[2], gfw[3]));
      }
    }
    __syncthreads();  // stage s consumed
    if (st.abort) break;
    if (tid == 0 && j + geo.stages < jend) {
      fence_proxy_async_smem();
      const int64_t jn = j + geo.stages;
      tma_issue<T, NIN>(geo, T_, D, smem + static_cast<size_t>(s) * geo.stage_bytes, &st.full[s], group_of(jn),
                        static_cast<int>(jn % geo.ns), base, rows);
    }
    if (p == geo.ns - 1) {
      // fold this token group's partial sums (all slices done)
      float v[L::kPad];
#pragma unroll
      for (int k = 0; k < L::kPad; ++k) v[k] = acc[k];
      warp_transpose_reduce<R>(v, lane);
#pragma unroll
      for (int r = 0; r < R; ++r) red[wid][lane * R + r] = v[r];
      __syncthreads();
      if (tok_ok) {
        for (int k = threadIdx.x; k < L::kAcc; k += blockDim.x) {
          float sum = 0.f;
          for (int w = 0; w < nw; ++w) sum += red[threadIdx.y * nw + w][k];
          if (k < N * N) {
            if (a.grad_phi) a.grad_phi[t * (N * N) + k] = sum;
          } else if constexpr (FUSED) {
            if (k < N * N + N) {
              if (a.grad_alpha) a.grad_alpha[t * N + (k - N * N)] = sum;
            } else {
              if (a.grad_beta) a.grad_beta[t * N + (k - N * N - N)] = sum;
            }
          }
          if constexpr (PROJ) fin[threadIdx.y][k] = sum;
        }
      }
      if constexpr (PROJ) {
        __syncthreads();
        if (tok_ok && a.grad_v != nullptr && threadIdx.x < N) {
          const int jj = threadIdx.x;
          const float* fr = fin[threadIdx.y];
          float ptr = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i) ptr = fmaf(phi[i * N + jj], fr[N * N + i], ptr);
          a.grad_v[t * N + jj] = (fr[N * N + jj] - ptr) + fr[N * N + N + jj];
        }
      }
      __syncthreads();  // red / fin reused by the next group
    }
  }
  if (st.abort) tma_drain(st, geo, j, jend);
}

// ================================================================= host side
// Rows per token that a stage holds.
inline int tma_rows(bool bwd, bool fused, int n) {
  if (!bwd) return fused ? n + 1 : 2 * n;
  return fused ? 2 * n + 2 : 2 * n;
}

// Tile geometry for D % chunk == 0 and 16-byte aligned bases; ok = false when
// the shape does not fit the pipeline (the element-wise kernels run instead).
inline bool tma_geometry(TmaGeometry& geo, bool bwd, bool fused, int n, int64_t T, int64_t D, int esize,
                         int num_sms) {
  const int E = 16 / esize;
  if (D % E != 0 || T <= 0 || D <= 0) return false;
  const int64_t nc = D / E;
  const int txmax = bwd ? 128 : 256;
  int tx = static_cast<int>(std::min<int64_t>(((nc + 31) / 32) * 32, txmax));
  const int64_t ns = (nc + tx - 1) / tx;
  geo.tx = tx;
  geo.ns = static_cast<int>(ns);
  geo.ds = tx * E;
  geo.pitch = ns == 1 ? static_cast<int>(D) : geo.ds;
  const int rows = tma_rows(bwd, fused, n);
  const int64_t tok_bytes = static_cast<int64_t>(rows) * geo.pitch * esize;
  const int64_t max_stage = bwd ? 48 * 1024 : 40 * 1024;
  int tok = max(1, kTmaMaxThreads / tx);
  if (tok > 16) tok = 16;
  while (tok > 1 && tok * tok_bytes > max_stage) --tok;
  if (tok_bytes > 96 * 1024) return false;
  if (tok > T) tok = static_cast<int>(T);
  geo.tok = tok;
  geo.stage_bytes = static_cast<int>(tok * tok_bytes);
  const int budget = 192 * 1024;
  int stages = budget / geo.stage_bytes;
  if (stages > 8) stages = 8;
  if (stages < 2) return false;
  geo.stages = stages;
  geo.smem_bytes = stages * geo.stage_bytes;
  geo.ngroups = (T + tok - 1) / tok;
  const int64_t grid = std::min<int64_t>(geo.ngroups, num_sms);
  geo.grid = static_cast<int>(grid);
  return tx * tok <= kTmaMaxThreads;
}

// Opt the kernel in to the dynamic shared memory it is launched with (a
// per-function attribute; cheap, and set on every launch so that every
// device and instantiation is covered).
template <typename KernelT>
inline int tma_prepare(KernelT* kernel, int smem_bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
    return HC_ERR_LAUNCH;
  return HC_OK;
}

template <typename T, typename P, bool FUSED, bool PROJ>
int launch_mix_fwd_tma(int n, const TmaGeometry& geo, const MixFwdArgs& a, cudaStream_t s) {
  const dim3 block(geo.tx, geo.tok, 1);
  switch (n) {
#define HC_CASE(NN)                                                                             \
  case NN: {                                                                                    \
    auto* k = mix_fwd_tma_kernel<T, P, NN, FUSED, PROJ>;                                       \
    if (int rc = tma_prepare(k, geo.smem_bytes)) return rc;                                     \
    k<<<geo.grid, block, geo.smem_bytes, s>>>(a, geo);                                \
    break;                                                                                      \
  }
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

template <typename T, typename P, bool FUSED, bool PROJ>
int launch_mix_bwd_tma(int n, const TmaGeometry& geo, const MixBwdArgs& a, cudaStream_t s) {
  const dim3 block(geo.tx, geo.tok, 1);
  switch (n) {
#define HC_CASE(NN)                                                                             \
  case NN: {                                                                                    \
    auto* k = mix_bwd_tma_kernel<T, P, NN, FUSED, PROJ>;                                       \
    if (int rc = tma_prepare(k, geo.smem_bytes)) return rc;                                     \
    k<<<geo.grid, block, geo.smem_bytes, s>>>(a, geo);                                \
    break;                                                                                      \
  }
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

// Per-dtype entry points of the pipelined kernels (mix_*.cu).
int mix_fwd_tma_f32(bool fused, bool proj, bool param_is_f32, int n, const TmaGeometry& g, const MixFwdArgs& a,
                    cudaStream_t s);
int mix_fwd_tma_f16(bool fused, bool proj, bool param_is_f32, int n, const TmaGeometry& g, const MixFwdArgs& a,
                    cudaStream_t s);
int mix_fwd_tma_bf16(bool fused, bool proj, bool param_is_f32, int n, const TmaGeometry& g, const MixFwdArgs& a,
                     cudaStream_t s);
int mix_bwd_tma_f32(bool fused, bool proj, bool param_is_f32, int n, const TmaGeometry& g, const MixBwdArgs& a,
                    cudaStream_t s);
int mix_bwd_tma_f16(bool fused, bool proj, bool param_is_f32, int n, const TmaGeometry& g, const MixBwdArgs& a,
                    cudaStream_t s);
int mix_bwd_tma_bf16(bool fused, bool proj, bool param_is_f32, int n, const TmaGeometry& g, const MixBwdArgs& a,
                     cudaStream_t s);
unsigned int mix_tma_take_timeouts_f32(bool reset);
unsigned int mix_tma_take_timeouts_f16(bool reset);
unsigned int mix_tma_take_timeouts_bf16(bool reset);

}  // namespace hc
