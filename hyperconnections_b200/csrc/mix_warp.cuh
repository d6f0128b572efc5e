// mix_warp.cuh — warp-specialised, TMA-fed stream-mixing kernels (fast path).
//
// A persistent CTA per SM owns a contiguous range of tokens and a ring of
// shared-memory stages, each with a "full" and an "empty" mbarrier. Warp 0 is
// the producer: one lane (four, in lockstep, for rings of small or sliced
// items) issues the bulk copies (plain cp.async.bulk into this CTA only) of
// the next token (or token-slice) into the next free stage with
// arrive.expect_tx on its full barrier. Warps 1..C are consumers: consumer c
// takes tokens c, c + C, ... of the range, waits on the stage's full barrier,
// computes in fp32 registers, stores 8-byte coalesced words to global memory,
// and releases the stage by arriving on its empty barrier. No CTA-wide
// barrier is needed in the steady state, consumers never issue copies, and
// stage indices and phases advance incrementally (no division per item).
//
// A stage holds one token-slice of every input row the kernel needs:
//   forward  fused: x (n rows), f (1)          add: x (n), Y (n)
//   backward fused: g_x (n), x (n), g_u (1), f (1)   add: g (n), x (n)
// laid out [tensor][row][pitch]. A token that fits one stage (the usual case)
// is ONE contiguous bulk copy per tensor; wider tokens are cut into slices,
// one copy per row slice, and the ring order interleaves the slices of the C
// tokens in flight so that every consumer always has its next slice coming.
//
// Lane l of a consumer reads W consecutive 32-bit words of every row at word
// offset seg*32*W + l*W (conflict-free shared-memory reads, coalesced global
// stores). A token stays on one consumer warp, so the backward's per-token
// sums (grad_Phi / grad_H, grad_alpha, grad_beta, the projection terms)
// accumulate in registers over all slices and fold with one warp
// transpose-reduce; at n >= 5 with sliced tokens or the projection the sums
// go to a per-warp Gram in shared memory a block of rows at a time (the
// blocked backward).
//
// Every wait is bounded (geo.wait_limit polls). A warp that gives up counts it
// in a device counter and in the library's status word (the next entry point
// call returns HC_ERR_TIMEOUT) and raises the CTA's abort flag; all warps
// stop, and before the CTA exits one thread waits (bounded again, always with
// the full kWaitPolls) for every copy the producer issued, so none lands after
// the CTA is gone.
#pragma once

#include <algorithm>
#include <cmath>
#include <type_traits>
#include <utility>

#include <cuda.h>  // CUtensorMap (the tensor maps are encoded through the runtime's driver entry point)
#include <cudaTypedefs.h>

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
// Tensor maps of the ring's inputs for tokens cut into slices (see
// ring_issue): one per input tensor, a 3-D view [rows][D / 64][64] of it.
struct alignas(64) RingMaps {
  CUtensorMap m[4];
};
constexpr int kTmaChunk = 64;  // elements in the innermost box dimension
// Swizzled stages of the tensor-core Gram path (see gram_mma_slice): each
// tensor's region is 1024-byte aligned (the 128-byte swizzle repeats every 8
// lines), and the ring's base is aligned up to 1024 bytes inside kSwzAlign
// bytes of slack.
constexpr int kSwzAlign = 1024;
__host__ __device__ constexpr int swz_region_bytes(int rows, int sl, int esize) {
  return (rows * sl * esize + kSwzAlign - 1) / kSwzAlign * kSwzAlign;
}
// Address of byte eb of a slice row (eb % 16 + access size <= 16) of row r in
// a swizzled region whose rows hold nc 128-byte lines each: line r * nc +
// eb / 128, its 16-byte unit (eb / 16) % 8 stored at unit
// ((eb / 16) % 8) ^ (line % 8).
__device__ __forceinline__ const uint8_t* swz_at(const uint8_t* region, int nc, int r, int eb) {
  const int off = r * nc * 128 + eb;  // line * 128 + byte in the line
  return region + (off ^ ((off >> 3) & 0x70));
}

// 3-D tensor copy global -> this CTA's shared memory through a tensor map in
// kernel-parameter space (no multicast; one destination CTA).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory (one destination CTA).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch. The ring kernels are launched with
// programmatic stream serialization allowed (launch_ring below). At entry a
// CTA lets the next kernel of the stream be scheduled (so that kernel's CTAs
// can take an SM the moment this kernel's CTA on it exits, and set up their
// rings while the rest of this grid finishes); after its own barrier setup it
// waits for the previous kernel of the stream to complete and flush before
// touching global memory. Both instructions are no-ops for a kernel launched
// without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

constexpr int kRingMaxStages = 32;  // stages of the per-CTA ring
constexpr int kWarpMaxWarps = 16;   // producer + consumers

// Count of bounded waits that gave up (one counter per translation unit; read
// and cleared by hc_wait_timeouts()).
static __device__ unsigned int g_mix_wait_timeouts;

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
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
  int consumers;    // consumer warps per CTA (one producer warp besides)
  int stages;       // stages of the CTA's ring
  int tpi;          // tokens per item (several small tokens share a stage)
  int sl;           // elements per slice
  int ns;           // slices per token (ns > 1 only with tpi == 1)
  int pitch;        // shared-memory row pitch (elements)
  int stage_bytes;  // rows * pitch * element size
  int grid;         // CTAs
  int smem_bytes;   // dynamic shared memory per CTA
  int producers;    // lanes of warp 0 that issue fills (1 <= producers <= stages)
  uint32_t wait_limit;  // polls of a data wait before it gives up
  unsigned int* status; // the library's status word (device-mapped host memory), or nullptr
  int tma;              // slices are copied through the tensor maps (ns > 1 only)
  int gram_mma;         // backward Gram on the tensor cores: 0 no, kGramPadded or kGramSwizzled stages
  int side;             // fused backward: g_u and f rows fetched by the consumers (side_fetch), not the ring
};


// Warps per CTA at most (producer included). The forward keeps 16 warps (128
// registers per thread) for n <= 4; the packed-pair backward for n <= 4 needs
// up to 170 registers, so 12 warps, and so does the blocked backward (tokens
// cut into slices at n >= 5); the backward of whole tokens at n = 7, 8 keeps
// all its sums in registers and runs 8 warps (255 registers).
constexpr int fwd_warp_cap(int n) { return n <= 4 ? 16 : 8; }
constexpr int bwd_warp_cap(int n, bool blocked) { return blocked || n <= 6 ? 12 : 8; }
constexpr int bwd_warp_cap_max() { return 12; }
constexpr int warp_cap(bool bwd, int n) { return bwd ? bwd_warp_cap_max() : fwd_warp_cap(n); }

// Issue the bulk copies of one item (cnt consecutive tokens, or one slice of
// one token) into a stage. Stage layout: [tensor][token][row][pitch].
// A slice through the tensor maps (geo.tma) is ONE 3-D tensor copy per
// tensor: box [rows][sl / 64][64] at (0, d0 / 64, t0 * rows), landing as
// [row][sl], the x coordinate always 0; the part of a short last slice past
// D is zero-filled and counted in the transaction bytes like the rest of the
// box. Otherwise a slice is one 1-D copy per row.
template <typename T, int NIN>
__device__ __forceinline__ void ring_issue(const WarpGeometry& geo, const RingMaps* maps, int64_t D,
                                           uint8_t* stage, uint64_t* bar, int64_t t0, int cnt, int p,
                                           const void* const* base, const int* rows) {
  constexpr int es = sizeof(T);
  const int64_t d0 = static_cast<int64_t>(p) * geo.sl;
  const int len = static_cast<int>(std::min<int64_t>(geo.sl, D - d0));
  int rtot = 0;
#pragma unroll
  for (int k = 0; k < NIN; ++k) rtot += rows[k];
  if (geo.tma) {
    mbar_expect_tx(bar, static_cast<uint32_t>(rtot * geo.sl * es));
    uint8_t* dst = stage;
#pragma unroll
    for (int k = 0; k < NIN; ++k) {
      tma_load_3d(dst, &maps->m[k], 0, static_cast<int>(d0 / kTmaChunk), static_cast<int>(t0 * rows[k]), bar);
      // swizzled stages: 1024-byte aligned regions
      dst += geo.gram_mma ? swz_region_bytes(rows[k], geo.sl, es) : static_cast<int>(rows[k]) * geo.pitch * es;
    }
    return;
  }
  mbar_expect_tx(bar, static_cast<uint32_t>(cnt * rtot * len * es));
  uint8_t* dst = stage;
#pragma unroll
  for (int k = 0; k < NIN; ++k) {
    const T* src = static_cast<const T*>(base[k]) + t0 * rows[k] * D;
    if (geo.ns == 1) {  // cnt whole tokens: contiguous in HBM
      bulk_g2s(dst, src, static_cast<uint32_t>(cnt * rows[k] * D * es), bar);
    } else {
      for (int r = 0; r < rows[k]; ++r)
        bulk_g2s(dst + static_cast<size_t>(r) * geo.pitch * es, src + r * D + d0, static_cast<uint32_t>(len * es),
                 bar);
    }
    dst += static_cast<size_t>(geo.tpi) * rows[k] * geo.pitch * es;
  }
}

// Shared-memory state of the ring.
struct RingState {
  uint64_t full[kRingMaxStages];
  uint64_t empty[kRingMaxStages];
  // Item index of the fill most recently started in each stage. A stage is
  // shared by items of different consumers in successive rounds, and a parity
  // wait can only tell adjacent phases apart: a consumer that reached item k
  // while item k - S (another consumer's) was still landing would see the
  // wrong phase as complete. Consumers therefore wait for tag == k first.
  volatile long long tag[kRingMaxStages];
  uint32_t last_parity[kRingMaxStages];
  int issued[kRingMaxStages];
  volatile int abort;
  alignas(16) uint32_t zrow[4];  // 16 zero bytes: the tensor-core Gram's rows past the matrix or the slice
};

__device__ __forceinline__ void ring_init(RingState& st, int stages) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&st.full[s], 1);
      mbar_init(&st.empty[s], 1);
      st.tag[s] = -1;
      st.issued[s] = 0;
      st.last_parity[s] = 0;
    }
    st.abort = 0;
    for (int i = 0; i < 4; ++i) st.zrow[i] = 0u;
    fence_mbar_init();
  }
  __syncthreads();
}

// Position of one item in the producer's sequence: unit group g0, slice p,
// unit w inside the group (Wg units in it), stage s with its fill parity ph,
// item index k.
struct ProducerCursor {
  int g0, p, w, Wg, s;
  uint32_t ph;
  int64_t k;
  __device__ __forceinline__ void step(int C, int ns, int nunits, int S) {
    if (++w == Wg) {
      w = 0;
      if (++p == ns) {
        p = 0;
        g0 += C;
        Wg = min(C, nunits - g0);
      }
    }
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
    ++k;
  }
};

// Producer loop, run by lanes 0 .. P - 1 of warp 0 (P = geo.producers).
// Work is cut into "units" (tpi consecutive tokens) dealt round-robin to the
// C consumers; units are issued in groups of C, slice-major inside a group, so
// consecutive items of one consumer are at most C apart and every consumer has
// its next item in flight. Item k goes to stage k mod S; a stage is reused
// once the consumer of item k - S has released it.
//
// One issuing thread fills a stage every ~250 ns whatever the copy size (a
// fixed cost per fill, measured on B200 with consumers that release at once),
// which caps 8 KB items near 4 TB/s. With P > 1, lane q issues items k = q,
// q + P, q + 2P, ...: the P lanes fill P consecutive items per round in
// lockstep. Within a round the P items sit in distinct stages (P <= S) and
// wait only on releases of items of earlier rounds, all issued, and every
// lane has seen the release of item k - 2S before it waits on the release of
// item k - S, so a parity wait can never mistake an older phase for the one
// it waits on.
#ifndef HC_GRID_STRIDE
#define HC_GRID_STRIDE 1  // build flag: units dealt to the CTAs grid-strided (1) or in contiguous ranges (0)
#endif

// The tokens of a CTA's units (tpi consecutive tokens each): unit u starts at
// token first + u * step, and the CTA's tokens end before `end`.
//
// Units are dealt to the CTAs grid-strided: global unit u * G + b goes to CTA
// b, so at any time the G CTAs stream neighbouring addresses of every tensor
// instead of G separate ranges. Measured on B200 against contiguous ranges
// (16,384 tokens, bf16, fused step): forward 43.0 -> 39.0-40.9 us at n = 4,
// D = 768, -5 to -9% at n = 2..8 over D = 512..4096; backward 0 to -3%;
// one loss, the n = 6, D = 512 forward (+4%).
struct UnitMap {
  int64_t first, step, end;
  int nunits;
  __device__ __forceinline__ int64_t tok(int u) const { return first + static_cast<int64_t>(u) * step; }
  __device__ __forceinline__ int cnt(int u, int tpi) const {
    return static_cast<int>(min(static_cast<int64_t>(tpi), end - tok(u)));
  }
};
__device__ __forceinline__ UnitMap unit_map(int64_t T, int tpi) {
  const int64_t G = gridDim.x, b = blockIdx.x;
  if (HC_GRID_STRIDE) {  // global unit u * G + b
    const int64_t nu = (T + tpi - 1) / tpi;
    return UnitMap{b * tpi, G * tpi, T, b < nu ? static_cast<int>((nu - 1 - b) / G + 1) : 0};
  }
  const int64_t t0 = T * b / G, t1 = T * (b + 1) / G;  // the CTA's contiguous range
  return UnitMap{t0, tpi, t1, static_cast<int>((t1 - t0 + tpi - 1) / tpi)};
}

template <typename T, int NIN>
__device__ __forceinline__ void ring_produce(RingState& st, const WarpGeometry& geo, uint8_t* smem, int64_t D,
                                             const UnitMap& um, const void* const* base,
                                             const int* rows, int lane, const RingMaps* maps = nullptr) {
  const int S = geo.stages, C = geo.consumers, P = geo.producers;
  const int nunits = um.nunits;
  if (P == 1) {
    int s = 0;
    uint32_t ph = 0;
    int64_t k = 0;
    for (int g0 = 0; g0 < nunits; g0 += C) {
      const int Wg = min(C, nunits - g0);
      for (int p = 0; p < geo.ns; ++p) {
        for (int w = 0; w < Wg; ++w) {
          if (st.abort) return;
          if (k >= S) {
            if (!warp_wait(&st.empty[s], ph ^ 1u, geo.wait_limit)) {
              report_timeout(&g_mix_wait_timeouts, geo.status);
              st.abort = 1;
              return;
            }
            fence_proxy_async_smem();
          }
          const int u = g0 + w;
          const int cnt = um.cnt(u, geo.tpi);
          ring_issue<T, NIN>(geo, maps, D, smem + static_cast<size_t>(s) * geo.stage_bytes, &st.full[s],
                             um.tok(u), cnt, p, base, rows);
          __threadfence_block();  // the arrive.expect_tx above is visible before the tag
          st.tag[s] = k;
          st.issued[s] = 1;
          st.last_parity[s] = ph;
          ++k;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
    return;
  }
  const unsigned mask = P >= 32 ? kFull : (1u << P) - 1u;
  ProducerCursor c{0, 0, 0, min(C, nunits), 0, 0u, 0};
  for (int i = 0; i < lane; ++i) c.step(C, geo.ns, nunits, S);
  while (true) {
    const bool act = c.g0 < nunits;
    if (!__any_sync(mask, act)) break;
    bool fail = false;
    if (act && !st.abort) {
      if (c.k >= S) {
        fail = !warp_wait(&st.empty[c.s], c.ph ^ 1u, geo.wait_limit);
        if (!fail) fence_proxy_async_smem();
      }
      if (!fail) {
        const int u = c.g0 + c.w;
        const int cnt = um.cnt(u, geo.tpi);
        ring_issue<T, NIN>(geo, maps, D, smem + static_cast<size_t>(c.s) * geo.stage_bytes, &st.full[c.s],
                           um.tok(u), cnt, c.p, base, rows);
        st.issued[c.s] = 1;
        st.last_parity[c.s] = c.ph;
        __threadfence_block();  // expect_tx and the drain record are visible before the tag
        st.tag[c.s] = c.k;
      }
    }
    if (fail) {
      report_timeout(&g_mix_wait_timeouts, geo.status);
      st.abort = 1;
    }
    if (__any_sync(mask, st.abort)) break;
    for (int i = 0; i < P; ++i) c.step(C, geo.ns, nunits, S);
  }
}

// Before the CTA exits: wait (bounded) for the last fill of every stage, so
// that no copy is still in flight (immediate in a normal run). The producer
// records each stage's last parity: computing it here would take two 64-bit
// divisions per stage on one thread, microseconds at the tail of every CTA.
__device__ __forceinline__ void ring_drain(RingState& st, int stages) {
  __syncthreads();
  if (threadIdx.x == 0)
    for (int s = 0; s < stages; ++s)
      if (st.issued[s]) warp_wait(&st.full[s], st.last_parity[s], kWaitPolls);
}

// Consumer-side cursor over the ring: item index k, its stage and parity.
struct RingCursor {
  int s;
  uint32_t ph;
  long long k;
  __device__ __forceinline__ void advance(int delta, int S) {
    k += delta;
    s += delta;
    if (s >= S) {
      s -= S;
      ph ^= 1u;
    }
  }
};

// Consumer wait for its item: first until the producer has started this
// item's fill (tag), then on the fill's phase. Bounded (`limit` polls each);
// warp-uniform result.
__device__ __forceinline__ bool ring_wait_item(RingState& st, const RingCursor& cur, uint32_t limit) {
  bool ok = false;
  for (uint32_t i = 0; i < limit; ++i) {
    if (st.tag[cur.s] == cur.k) {
      ok = true;
      break;
    }
    if (st.abort) break;
    __nanosleep(32);
  }
  __threadfence_block();
  if (ok) ok = warp_wait(&st.full[cur.s], cur.ph, limit);
  return __all_sync(kFull, ok);
}

// Per-token parameters in registers.
template <typename P, int N, bool FUSED, bool PROJ>
struct TokParams {
  float phi[N * N];
  float vv[PROJ ? N : 1], cc[PROJ ? N : 1];
  float al[FUSED ? N : 1], be[FUSED ? N : 1];
  __device__ __forceinline__ void load(const void* phi_p, const void* v_p, const float* alpha, const float* beta,
                                       int64_t t) {
    load_params_keep<P, N * N>(static_cast<const P*>(phi_p) + t * (N * N), phi);
    if constexpr (PROJ) {
      load_params_keep<P, N>(static_cast<const P*>(v_p) + t * N, vv);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float pv = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) pv = fmaf(phi[i * N + j], vv[j], pv);
        cc[i] = vv[i] - pv;
      }
    }
    if constexpr (FUSED) {
      load_params_keep<float, N>(alpha + t * N, al);
      load_params_keep<float, N>(beta + t * N, be);
    }
  }
};

// ------------------------------------------------------------ packed pairs
// For n <= 4 the kernels run on pairs of elements with fma.rn.f32x2
// (__ffma2_rn): two independent fp32 FMAs per instruction on a register pair,
// with the per-token parameters duplicated into pairs. A 32-bit word of
// bf16/fp16 holds exactly one pair; fp32 streams pair two consecutive words.
// Every element still sees one fp32 FMA per term, in the same order.
constexpr bool use_pairs(int n) { return n <= 4; }

__device__ __forceinline__ float2 dup2(float v) { return make_float2(v, v); }

template <typename T> struct PairIO;
template <> struct PairIO<__nv_bfloat16> {
  static constexpr int WORDS = 1;
  __device__ static __forceinline__ float2 get(const uint32_t* w) {
    return make_float2(__uint_as_float(w[0] << 16), __uint_as_float(w[0] & 0xffff0000u));
  }
  __device__ static __forceinline__ void put(float2 v, uint32_t* w) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    w[0] = *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct PairIO<__half> {
  static constexpr int WORDS = 1;
  __device__ static __forceinline__ float2 get(const uint32_t* w) {
    __half2 h = *reinterpret_cast<const __half2*>(w);
    return __half22float2(h);
  }
  __device__ static __forceinline__ void put(float2 v, uint32_t* w) {
    __half2 h = __floats2half2_rn(v.x, v.y);
    w[0] = *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct PairIO<float> {
  static constexpr int WORDS = 2;
  __device__ static __forceinline__ float2 get(const uint32_t* w) {
    return make_float2(__uint_as_float(w[0]), __uint_as_float(w[1]));
  }
  __device__ static __forceinline__ void put(float2 v, uint32_t* w) {
    w[0] = __float_as_uint(v.x);
    w[1] = __float_as_uint(v.y);
  }
};

template <typename P, int N, bool FUSED, bool PROJ>
struct TokParams2 {
  float2 phi[N * N];
  float2 vv[PROJ ? N : 1], nvv[PROJ ? N : 1], cc[PROJ ? N : 1];
  float2 al[FUSED ? N : 1], be[FUSED ? N : 1];
  __device__ __forceinline__ void load(const void* phi_p, const void* v_p, const float* alpha, const float* beta,
                                       int64_t t) {
    TokParams<P, N, FUSED, PROJ> s;
    s.load(phi_p, v_p, alpha, beta, t);
#pragma unroll
    for (int k = 0; k < N * N; ++k) phi[k] = dup2(s.phi[k]);
    if constexpr (PROJ) {
#pragma unroll
      for (int k = 0; k < N; ++k) {
        vv[k] = dup2(s.vv[k]);
        nvv[k] = dup2(-s.vv[k]);
        cc[k] = dup2(s.cc[k]);
      }
    }
    if constexpr (FUSED) {
#pragma unroll
      for (int k = 0; k < N; ++k) {
        al[k] = dup2(s.al[k]);
        be[k] = dup2(s.be[k]);
      }
    }
  }
};

template <typename T, typename P, int N, bool FUSED, bool PROJ, int W>
__device__ __forceinline__ void fwd_slice2(const MixFwdArgs& a, const TokParams2<P, N, FUSED, PROJ>& pr,
                                           const uint8_t* xsb, const uint8_t* ssb, int pitch, int64_t t, int64_t d0,
                                           int len, int lane) {
  using IO = PairIO<T>;
  constexpr int K = Word<T>::K;
  constexpr int WP = IO::WORDS;
  constexpr int NS = FUSED ? 1 : N;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  static_assert(W % WP == 0, "lane access must hold whole pairs");
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* ot = static_cast<T*>(a.out) + t * N * D + d0;
  T* ut = FUSED ? static_cast<T*>(a.u) + t * D + d0 : nullptr;
  const float2 zero = make_float2(0.f, 0.f);
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> xw[N], sw[NS];
#pragma unroll
    for (int j = 0; j < N; ++j) xw[j] = lds_words<W>(xsb + eo + j * rowb);
#pragma unroll
    for (int i2 = 0; i2 < NS; ++i2) sw[i2] = lds_words<W>(ssb + eo + i2 * rowb);
    uint32_t ow[N][W], uw[W];
#pragma unroll
    for (int w = 0; w < W; w += WP) {
      float2 x[N], sv[NS];
#pragma unroll
      for (int j = 0; j < N; ++j) x[j] = IO::get(&xw[j].w[w]);
#pragma unroll
      for (int i2 = 0; i2 < NS; ++i2) sv[i2] = IO::get(&sw[i2].w[w]);
      float2 av = zero;
      if constexpr (PROJ) {
#pragma unroll
        for (int j = 0; j < N; ++j) av = __ffma2_rn(pr.vv[j], x[j], av);
      }
      if constexpr (FUSED) {
        float2 u = zero;
#pragma unroll
        for (int j = 0; j < N; ++j) u = __ffma2_rn(pr.al[j], x[j], u);
        IO::put(u, &uw[w]);
      }
#pragma unroll
      for (int i2 = 0; i2 < N; ++i2) {
        float2 o = zero;
#pragma unroll
        for (int j = 0; j < N; ++j) o = __ffma2_rn(pr.phi[i2 * N + j], x[j], o);
        if constexpr (PROJ) o = __ffma2_rn(pr.cc[i2], av, o);
        if constexpr (FUSED) {
          o = __ffma2_rn(pr.be[i2], sv[0], o);
        } else {
          o = __fadd2_rn(o, sv[i2]);
        }
        IO::put(o, &ow[i2][w]);
      }
    }
#pragma unroll
    for (int i2 = 0; i2 < N; ++i2) stg_words<W>(ot + i2 * D + e0, ow[i2]);
    if constexpr (FUSED) stg_words<W>(ut + e0, uw);
  }
}

template <typename T, typename P, int N, bool FUSED, bool PROJ, int W>
__device__ __forceinline__ void bwd_slice2(const MixBwdArgs& a, const TokParams2<P, N, FUSED, PROJ>& pr,
                                           float2* acc, const uint8_t* gsb, const uint8_t* xsb, const uint8_t* usb,
                                           const uint8_t* fsb, int pitch, int64_t t, int64_t d0, int len,
                                           int lane) {
  using IO = PairIO<T>;
  constexpr int K = Word<T>::K;
  constexpr int WP = IO::WORDS;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  static_assert(W % WP == 0, "lane access must hold whole pairs");
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * N * D + d0 : nullptr;
  T* gft = (FUSED && a.grad_f) ? static_cast<T*>(a.grad_f) + t * D + d0 : nullptr;
  const float2 zero = make_float2(0.f, 0.f);
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> gwr[N], xwr[N], uwr, fwr;
#pragma unroll
    for (int r = 0; r < N; ++r) gwr[r] = lds_words<W>(gsb + eo + r * rowb);
#pragma unroll
    for (int r = 0; r < N; ++r) xwr[r] = lds_words<W>(xsb + eo + r * rowb);
    if constexpr (FUSED) {
      uwr = lds_words<W>(usb + eo);
      fwr = lds_words<W>(fsb + eo);
    }
    uint32_t gxo[N][W], gfo[W];
#pragma unroll
    for (int w = 0; w < W; w += WP) {
      float2 g[N], x[N], gu = zero, f = zero;
#pragma unroll
      for (int r = 0; r < N; ++r) g[r] = IO::get(&gwr[r].w[w]);
#pragma unroll
      for (int r = 0; r < N; ++r) x[r] = IO::get(&xwr[r].w[w]);
      if constexpr (FUSED) {
        gu = IO::get(&uwr.w[w]);
        f = IO::get(&fwr.w[w]);
      }
      float2 av = zero, bt = zero;
      if constexpr (PROJ) {
#pragma unroll
        for (int j = 0; j < N; ++j) av = __ffma2_rn(pr.vv[j], x[j], av);
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) bt = __ffma2_rn(g[i2], pr.cc[i2], bt);
      }
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float2 o = zero;
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) o = __ffma2_rn(pr.phi[i2 * N + j], g[i2], o);
        if constexpr (PROJ) o = __ffma2_rn(pr.vv[j], bt, o);
        if constexpr (FUSED) o = __ffma2_rn(pr.al[j], gu, o);
        IO::put(o, &gxo[j][w]);
      }
      if constexpr (FUSED) {
        float2 o = zero;
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) o = __ffma2_rn(pr.be[i2], g[i2], o);
        IO::put(o, &gfo[w]);
      }
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float2 xv = x[j];
        if constexpr (PROJ) xv = __ffma2_rn(pr.nvv[j], av, xv);  // x_eff = x - v (v^T x)
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) acc[i2 * N + j] = __ffma2_rn(g[i2], xv, acc[i2 * N + j]);
      }
      if constexpr (FUSED) {
#pragma unroll
        for (int j = 0; j < N; ++j) acc[N * N + j] = __ffma2_rn(gu, x[j], acc[N * N + j]);
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) acc[N * N + N + i2] = __ffma2_rn(g[i2], f, acc[N * N + N + i2]);
      }
      if constexpr (PROJ) {
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) acc[N * N + i2] = __ffma2_rn(g[i2], av, acc[N * N + i2]);
#pragma unroll
        for (int j = 0; j < N; ++j) acc[N * N + N + j] = __ffma2_rn(bt, x[j], acc[N * N + N + j]);
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
}

// ================================================================= forward
template <typename T, typename P, int N, bool FUSED, bool PROJ, int W>
__device__ __forceinline__ void fwd_slice(const MixFwdArgs& a, const TokParams<P, N, FUSED, PROJ>& pr,
                                          const uint8_t* xsb, const uint8_t* ssb, int pitch, int64_t t, int64_t d0,
                                          int len, int lane) {
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int NS = FUSED ? 1 : N;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* ot = static_cast<T*>(a.out) + t * N * D + d0;
  T* ut = FUSED ? static_cast<T*>(a.u) + t * D + d0 : nullptr;
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> xw[N], sw[NS];
#pragma unroll
    for (int j = 0; j < N; ++j) xw[j] = lds_words<W>(xsb + eo + j * rowb);
#pragma unroll
    for (int i2 = 0; i2 < NS; ++i2) sw[i2] = lds_words<W>(ssb + eo + i2 * rowb);
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
}

template <typename T, typename P, int N, bool FUSED, bool PROJ, int W>
__global__ void __launch_bounds__(fwd_warp_cap(N) * 32, 1)
mix_fwd_warp_kernel(const MixFwdArgs a, const WarpGeometry geo, const __grid_constant__ RingMaps maps) {
  constexpr int NS = FUSED ? 1 : N;
  constexpr int es = sizeof(T);
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
  const uint32_t xregion = static_cast<uint32_t>(geo.tpi) * N * rowb;  // bytes of the x rows of a stage
  const bool single = geo.tpi == 1;

  if (warp == 0) {
    if (lane < geo.producers) {
      const void* base[2] = {a.x, a.src};
      const int rows[2] = {N, NS};
      ring_produce<T, 2>(st, geo, smem, D, um, base, rows, lane, &maps);
    }
  } else if (warp - 1 < C) {
    const int c = warp - 1;
    using Params = std::conditional_t<use_pairs(N), TokParams2<P, N, FUSED, PROJ>, TokParams<P, N, FUSED, PROJ>>;
    Params pr;
    RingCursor cur{c, 0u, c};
    for (int g0 = 0; g0 < nunits; g0 += C) {
      const int Wg = min(C, nunits - g0);
      if (c >= Wg) break;
      const int u = g0 + c;
      const int cnt = um.cnt(u, geo.tpi);
      const int64_t t0 = um.tok(u);
      pr.load(a.phi, a.v, a.alpha, a.beta, t0);  // overlaps the wait for the data
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
        if (single) {  // one token (or slice) per item: the common, hottest path
          if constexpr (use_pairs(N)) {
            fwd_slice2<T, P, N, FUSED, PROJ, W>(a, pr, sb, sb + N * rowb, geo.pitch, t0, d0, len, lane);
          } else {
            fwd_slice<T, P, N, FUSED, PROJ, W>(a, pr, sb, sb + N * rowb, geo.pitch, t0, d0, len, lane);
          }
        } else {
          for (int tt = 0; tt < cnt; ++tt) {
            const int64_t t = t0 + tt;
            if (tt > 0) pr.load(a.phi, a.v, a.alpha, a.beta, t);
            const uint8_t* xs = sb + tt * N * rowb;
            const uint8_t* ss = sb + xregion + tt * NS * rowb;
            if constexpr (use_pairs(N)) {
              fwd_slice2<T, P, N, FUSED, PROJ, W>(a, pr, xs, ss, geo.pitch, t, d0, len, lane);
            } else {
              fwd_slice<T, P, N, FUSED, PROJ, W>(a, pr, xs, ss, geo.pitch, t, d0, len, lane);
            }
          }
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

// ================================================================= backward
template <typename T, typename P, int N, bool FUSED, bool PROJ, int W>
__device__ __forceinline__ void bwd_slice(const MixBwdArgs& a, const TokParams<P, N, FUSED, PROJ>& pr,
                                          float* acc, const uint8_t* gsb, const uint8_t* xsb, const uint8_t* usb,
                                          const uint8_t* fsb, int pitch, int64_t t, int64_t d0, int len, int lane) {
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * N * D + d0 : nullptr;
  T* gft = (FUSED && a.grad_f) ? static_cast<T*>(a.grad_f) + t * D + d0 : nullptr;
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> gw_[N], xw[N], uw, fw;
#pragma unroll
    for (int r = 0; r < N; ++r) gw_[r] = lds_words<W>(gsb + eo + r * rowb);
#pragma unroll
    for (int r = 0; r < N; ++r) xw[r] = lds_words<W>(xsb + eo + r * rowb);
    if constexpr (FUSED) {
      uw = lds_words<W>(usb + eo);
      fw = lds_words<W>(fsb + eo);
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
}

__device__ __forceinline__ float phi_of(float v) { return v; }
__device__ __forceinline__ float phi_of(float2 v) { return v.x; }

// Fold the 32 lanes' partial sums of one token and write its parameter
// gradients (and grad_v for the projection).
template <typename P, int N, bool FUSED, bool PROJ, typename Params>
__device__ __forceinline__ void bwd_finish(const MixBwdArgs& a, const Params& pr, const float* acc, int64_t t,
                                           int lane) {
  using L = BwdLayout<N, FUSED, PROJ>;
  constexpr int R = L::kR;
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
          for (int i2 = 0; i2 < N; ++i2) ptr = fmaf(phi_of(pr.phi[i2 * N + j]), rho[i2], ptr);
          out = (rho[j] - ptr) + bp[j];
        }
      }
      a.grad_v[t * N + lane] = out;
    }
  }
}

// Side rows of the fused backward (geo.side): instead of two small bulk
// copies per item (a bulk copy has a fixed cost, and the g_u / f rows of one
// token are 1.5 KB at D = 768), each consumer warp copies the g_u and f rows
// of its next unit (cnt consecutive tokens: contiguous in HBM) into one of
// two slots of its own with 16-byte cp.async while it computes the current
// unit. Slot layout: [g_u rows of tpi tokens][f rows of tpi tokens], D
// elements a row. The ring then carries the 2n rows of g and x.
template <typename T>
__device__ __forceinline__ void side_fetch(uint8_t* slot, const MixBwdArgs& a, int64_t t0, int cnt, int tpi,
                                           int lane) {
  const int64_t rowb = a.D * static_cast<int64_t>(sizeof(T));
  const int chunks = static_cast<int>(cnt * rowb / 16);
  const uint8_t* gu = static_cast<const uint8_t*>(a.gu) + t0 * rowb;
  const uint8_t* f = static_cast<const uint8_t*>(a.f) + t0 * rowb;
  uint8_t* fslot = slot + tpi * rowb;
  for (int i = lane; i < chunks; i += 32) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(slot + i * 16)), "l"(gu + i * 16)
                 : "memory");
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(fslot + i * 16)), "l"(f + i * 16)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// ------------------------------------------- blocked backward for n >= 5
// With n >= 5 the per-lane sums of the backward (n^2 + 2n of them) and Phi
// together no longer leave room for 12 warps. The blocked path splits each
// slice's work instead:
//   pass A  grad_x (and grad_f) of the slice, no sums;
//   pass B  the slice's Gram sums, a block of rows at a time: a block fills
//           at most 32 sums per lane, one warp transpose-reduce leaves one sum
//           per lane, and that lane adds it into the warp's Gram in shared
//           memory;
//   finish  at the token's last slice, the parameter gradients from the Gram.
// The Gram is M = A B^T over the slice's elements, with A's rows g_0..g_{n-1}
// and B's rows x_0..x_{n-1}, each extended by g_u and f in the fused step.
// Then grad_Phi_ij = M_ij, and in the fused step grad_alpha_j = M_nj and
// grad_beta_i = M_in; with the projection (stream_mix_add with v) the finish
// forms its terms from M alone (bwd_gram_finish).
// The blocked path runs at n >= 5 for tokens cut into slices, and for every
// token with the projection (whose extra sums the finish derives from the
// plain Gram). Measured on B200: +1-7% for sliced tokens; with the projection
// +3-17% over the single pass (which spills at n = 6, 8), except -1.5% at
// n = 7, D = 768; for whole tokens without the projection the single pass
// with every sum in registers stays faster (by 16% at n = 8, D = 512).
constexpr bool bwd_blocked_n(int n) { return n >= 5; }
inline bool bwd_blocked(int n, bool proj, int ns) { return bwd_blocked_n(n) && (ns > 1 || proj); }

template <int N, bool FUSED>
struct GramShape {
  static constexpr bool EXTRA = FUSED;
  static constexpr int NA = N + (EXTRA ? 1 : 0);  // rows (and columns) of M
  static constexpr int SIZE = NA * NA;
  static constexpr int RB = 32 / NA;              // rows per block: RB * NA <= 32 sums
};

// Pass A: grad_x_j = sum_i Phi_ij g_i (+ v_j c^T g) (+ alpha_j g_u) and
// grad_f = beta^T g over one slice; same arithmetic as bwd_slice.
#ifndef HC_PASSA_PAIRS
#define HC_PASSA_PAIRS 1  // build flag: 0 runs pass A's grad_x as scalar FMA chains (measurements)
#endif

// SWZ: the stage's g and g_u regions are chunk-major swizzled (the tensor-core
// Gram path, W == 1: a segment is one 64-element chunk); otherwise row-major
// with `pitch` elements per row.
template <typename T, typename P, int N, bool FUSED, bool PROJ, int W, bool SWZ = false>
__device__ __forceinline__ void bwd_grads_slice(const MixBwdArgs& a, const TokParams<P, N, FUSED, PROJ>& pr,
                                                const uint8_t* gsb, const uint8_t* usb, int pitch, int64_t t,
                                                int64_t d0, int len, int lane, int nc = 0) {
  static_assert(!SWZ || (W <= 2 && sizeof(T) == 2), "swizzled stages: 4- or 8-byte lane reads of 2-byte elements");
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  const int64_t D = a.D;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * N * D + d0 : nullptr;
  T* gft = (FUSED && a.grad_f) ? static_cast<T*>(a.grad_f) + t * D + d0 : nullptr;
  if (gxt == nullptr && gft == nullptr) return;
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> gw_[N], uw;
    if constexpr (SWZ) {
#pragma unroll
      for (int r = 0; r < N; ++r) gw_[r] = lds_words<W>(swz_at(gsb, nc, r, static_cast<int>(eo)));
      if constexpr (FUSED) uw = lds_words<W>(swz_at(usb, nc, 0, static_cast<int>(eo)));
    } else {
#pragma unroll
      for (int r = 0; r < N; ++r) gw_[r] = lds_words<W>(gsb + eo + r * rowb);
      if constexpr (FUSED) uw = lds_words<W>(usb + eo);
    }
    uint32_t gxo[N][W], gfo[W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      float ge[N][K], gue[K];
#pragma unroll
      for (int r = 0; r < N; ++r) Wd::get(gw_[r].w[w], ge[r]);
      if constexpr (FUSED) Wd::get(uw.w[w], gue);
      float bt[K];
      if constexpr (PROJ) {
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i2 = 0; i2 < N; ++i2) s = fmaf(ge[i2][e], pr.cc[i2], s);
          bt[e] = s;
        }
      }
      // grad_x on packed pairs of output rows (j, j + 1): fma.rn.f32x2 of the
      // pair (Phi_ij, Phi_i,j+1) with g_i duplicated, two fp32 FMAs per
      // instruction with each output seeing the same terms in the same order
      // as one FMA chain; an odd last row runs alone.
      constexpr int JP = HC_PASSA_PAIRS ? N / 2 : 0;
      float2 op[JP > 0 ? JP : 1][K];
#pragma unroll
      for (int e = 0; e < K; ++e) {
        float2 gg[N];
#pragma unroll
        for (int i2 = 0; i2 < N; ++i2) gg[i2] = dup2(ge[i2][e]);
#pragma unroll
        for (int k = 0; k < JP; ++k) {
          float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int i2 = 0; i2 < N; ++i2)
            s2 = __ffma2_rn(make_float2(pr.phi[i2 * N + 2 * k], pr.phi[i2 * N + 2 * k + 1]), gg[i2], s2);
          if constexpr (PROJ) s2 = __ffma2_rn(make_float2(pr.vv[2 * k], pr.vv[2 * k + 1]), dup2(bt[e]), s2);
          if constexpr (FUSED) s2 = __ffma2_rn(make_float2(pr.al[2 * k], pr.al[2 * k + 1]), dup2(gue[e]), s2);
          op[k][e] = s2;
        }
      }
#pragma unroll
      for (int k = 0; k < JP; ++k) {
        float lo[K], hi[K];
#pragma unroll
        for (int e = 0; e < K; ++e) {
          lo[e] = op[k][e].x;
          hi[e] = op[k][e].y;
        }
        gxo[2 * k][w] = Wd::put(lo);
        gxo[2 * k + 1][w] = Wd::put(hi);
      }
#pragma unroll
      for (int j = 2 * JP; j < N; ++j) {
        float o[K];
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i2 = 0; i2 < N; ++i2) s = fmaf(pr.phi[i2 * N + j], ge[i2][e], s);
          if constexpr (PROJ) s = fmaf(pr.vv[j], bt[e], s);
          if constexpr (FUSED) s = fmaf(pr.al[j], gue[e], s);
          o[e] = s;
        }
        gxo[j][w] = Wd::put(o);
      }
      if constexpr (FUSED) {
        float o[K];
#pragma unroll
        for (int e = 0; e < K; ++e) {
          float s = 0.f;
#pragma unroll
          for (int i2 = 0; i2 < N; ++i2) s = fmaf(pr.be[i2], ge[i2][e], s);
          o[e] = s;
        }
        gfo[w] = Wd::put(o);
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
}

// Pass B for the rows [R0, R0 + RB) of M over one slice, added into the
// warp's Gram (row-major, NA x NA, in shared memory). Lane l owns entry
// R0 * NA + l of the block, in every slice, so its read-modify-write needs no
// synchronisation.
template <typename T, int N, bool FUSED, int W, int R0>
__device__ __forceinline__ void bwd_gram_block(float* gram, const uint8_t* gsb, const uint8_t* xsb,
                                               const uint8_t* usb, const uint8_t* fsb, int pitch, int len,
                                               int lane) {
  using G = GramShape<N, FUSED>;
  using Wd = Word<T>;
  constexpr int K = Wd::K;
  constexpr int es = sizeof(T);
  constexpr int SEGW = 32 * W * K;
  constexpr int NA = G::NA;
  constexpr int RB = G::RB < NA - R0 ? G::RB : NA - R0;
  constexpr bool HAS_EXTRA = G::EXTRA && R0 + RB > N;  // the block ends with row n of M (g_u)
  constexpr int RG = HAS_EXTRA ? RB - 1 : RB;          // g rows of the block
  constexpr int NGW = RG > 0 ? RG : 1;
  const uint32_t rowb = static_cast<uint32_t>(pitch) * es;
  float acc[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) acc[k] = 0.f;
  for (int e0 = lane * W * K; e0 < len; e0 += SEGW) {
    const uint32_t eo = static_cast<uint32_t>(e0) * es;
    Words<W> xw[N], fw, gw[NGW], uw;
#pragma unroll
    for (int j = 0; j < N; ++j) xw[j] = lds_words<W>(xsb + eo + j * rowb);
    if constexpr (FUSED) fw = lds_words<W>(fsb + eo);
#pragma unroll
    for (int r = 0; r < RG; ++r) gw[r] = lds_words<W>(gsb + eo + (R0 + r) * rowb);
    if constexpr (HAS_EXTRA) uw = lds_words<W>(usb + eo);
#pragma unroll
    for (int w = 0; w < W; ++w) {
      float col[NA][K], row[RB][K];
#pragma unroll
      for (int j = 0; j < N; ++j) Wd::get(xw[j].w[w], col[j]);
      if constexpr (FUSED) Wd::get(fw.w[w], col[N]);
#pragma unroll
      for (int r = 0; r < RG; ++r) Wd::get(gw[r].w[w], row[r]);
      if constexpr (HAS_EXTRA) Wd::get(uw.w[w], row[RG]);
#pragma unroll
      for (int e = 0; e < K; ++e) {
#pragma unroll
        for (int r = 0; r < RB; ++r) {
#pragma unroll
          for (int j = 0; j < NA; ++j) {
            if (R0 + r == N && j == N) continue;  // M_nn is not used
            acc[r * NA + j] = fmaf(row[r][e], col[j][e], acc[r * NA + j]);
          }
        }
      }
    }
  }
  warp_transpose_reduce<1>(acc, lane);  // lane l: the warp's sum of entry l
  if (lane < RB * NA) gram[R0 * NA + lane] += acc[0];
}

template <typename T, int N, bool FUSED, int W, int R0>
__device__ __forceinline__ void bwd_gram_slice(float* gram, const uint8_t* gsb, const uint8_t* xsb,
                                               const uint8_t* usb, const uint8_t* fsb, int pitch, int len,
                                               int lane) {
  using G = GramShape<N, FUSED>;
  if constexpr (R0 < G::NA) {
    bwd_gram_block<T, N, FUSED, W, R0>(gram, gsb, xsb, usb, fsb, pitch, len, lane);
    bwd_gram_slice<T, N, FUSED, W, R0 + G::RB>(gram, gsb, xsb, usb, fsb, pitch, len, lane);
  }
}

// ------------------------------------- pass B on the tensor cores (bf16 / fp16)
// For half-precision streams the slice's Gram M = A B^T (A = [g; g_u] rows, B
// = [x; f] rows, K = the slice's elements) is a warp-level contraction:
// ldmatrix loads the rows straight from the ring stage and
// mma.sync.m16n8k16 (fp32 accumulation; the product of two bf16 / fp16 values
// is exact in fp32) accumulates a 16 x 8 tile per instruction, one or two
// tiles for NA <= 8 or 9 columns. Rows and columns past NA, and the second
// half of a 16-element step past the slice's end (slices are multiples of 8
// elements), read the ring's zeroed 16-byte row. The accumulators stay in
// registers over all slices of the token; at its last slice they are written
// to the warp's Gram, whose finish is the CUDA-core path's.
//
// Stage layouts of this path. An 8 x 8 ldmatrix reads the same 16 bytes of 8
// rows; in the plain row-major stage the rows are a multiple of 128 bytes
// apart and all eight sit in the same four banks (an 8-way conflict). Two
// layouts avoid it:
//   kGramSwizzled  one TMA tensor copy per tensor and slice with the 128-byte
//                  swizzle, box [rows][sl / 64][64] as in the plain ring: a
//                  tensor's region (1024-byte aligned) holds row r's chunk c
//                  in 128-byte line L = r * nc + c (nc = sl / 64), its 16-byte
//                  unit u at unit u ^ (L mod 8). Slices hold an odd number of
//                  chunks, so the 8 rows of one chunk fall in 8 different
//                  unit positions; a warp reading one line 4 bytes a lane
//                  (pass A) still touches all 32 banks once. The part of the
//                  last slice past D is zero-filled by the copy.
//   kGramPadded    one bulk copy per row into rows padded by 16 bytes (pitch
//                  sl + 8 elements): row r starts 4 r banks further.
// Measured on B200 (fused backward, 16,384 tokens, bf16): the swizzled ring
// is faster at even n (n = 8, D = 1024: 190 against 225 us; n = 6, D = 1024:
// 147 against 179 us; within 1.5% at D = 2048, 4096), the padded one at odd
// n (n = 7, D = 1536: 249 against 307 us; n = 5, D = 2048: 236 against
// 311 us, where odd chunk counts make 28 KB stages and fewer consumers).
template <typename T> struct MmaKind;
template <> struct MmaKind<__nv_bfloat16> {
  __device__ static __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct MmaKind<__half> {
  __device__ static __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
#ifndef HC_GRAM_MMA
#define HC_GRAM_MMA 1  // build flag: 0 keeps pass B on the FMA pipe for every dtype (measurements)
#endif
constexpr bool gram_mma_dtype(int esize) { return HC_GRAM_MMA && esize == 2; }
constexpr int kGramPadded = 1;    // geo.gram_mma: row copies into 16-byte padded rows
constexpr int kGramSwizzled = 2;  // geo.gram_mma: swizzled TMA tensor copies
constexpr int kGramPad = 8;       // elements of padding per row of kGramPadded stages
constexpr int kGramBudget = 216 * 1024;  // bytes of ring stages of the tensor-core Gram backward


__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

template <int N, bool FUSED>
struct GramMma {
  static constexpr int NA = N + (FUSED ? 1 : 0);
  static constexpr int NT = (NA + 7) / 8;  // n8 tiles of columns
};

// Address of byte eb of row r of a stage region: swizzled (nc lines a row)
// or row-major with rowb bytes a row.
template <bool SWZ>
__device__ __forceinline__ const uint8_t* stage_at(const uint8_t* region, uint32_t rowb, int nc, int r, int eb) {
  if constexpr (SWZ) {
    return swz_at(region, nc, r, eb);
  } else {
    return region + r * rowb + eb;
  }
}

// Accumulates one slice of a Gram M = A B^T into c (see above): A's rows are
// A0 rows of region a0 then A1 rows of region a1 (at most 16), B's rows B0
// rows of region b0 then B1 rows of region b1 (at most 16, (B0 + B1 + 7) / 8
// tiles of 8 columns); rows past them read zrow (16 zero bytes in shared
// memory). Padded stages: rowb bytes a row, and the second half of a
// 16-element step past the slice's end (slices are multiples of 8 elements)
// reads zrow; swizzled stages: nc lines a row, the box zero-filled past D.
template <typename T, int A0, int A1, int B0, int B1, bool SWZ>
__device__ __forceinline__ void gram_mma_slice(float (&c)[(B0 + B1 + 7) / 8][4], const uint8_t* a0,
                                               const uint8_t* a1, const uint8_t* b0, const uint8_t* b1,
                                               const uint8_t* zrow, uint32_t rowb, int nc, int len, int lane) {
  constexpr int NT = (B0 + B1 + 7) / 8;
  static_assert(A0 + A1 <= 16 && NT <= 2, "one 16-row A tile, at most two 8-column B tiles");
  constexpr int es = sizeof(T);
  const int q = lane >> 3;
  // A: matrix q holds rows (q & 1) * 8 + (lane & 7), elements (q >> 1) * 8 + [0, 8)
  const int ar = (q & 1) * 8 + (lane & 7);
  const uint8_t* areg = ar < A0 ? a0 : (ar < A0 + A1 ? a1 : nullptr);
  const int arow = ar < A0 ? ar : ar - A0;
  const int akof = (q >> 1) * 8;
  // B: matrix q holds rows (columns of M) (q >> 1) * 8 + (lane & 7), elements (q & 1) * 8 + [0, 8)
  const int bj = (q >> 1) * 8 + (lane & 7);
  const uint8_t* breg = bj < B0 ? b0 : (bj < B0 + B1 ? b1 : nullptr);
  const int brow = bj < B0 ? bj : bj - B0;
  const int bkof = (q & 1) * 8;
  const uint32_t z = smem_u32(zrow);
  for (int k0 = 0; k0 < len; k0 += 16) {
    const bool ain = areg && (SWZ || k0 + akof < len), bin = breg && (SWZ || k0 + bkof < len);
    const uint32_t aaddr = ain ? smem_u32(stage_at<SWZ>(areg, rowb, nc, arow, (k0 + akof) * es)) : z;
    const uint32_t baddr = bin ? smem_u32(stage_at<SWZ>(breg, rowb, nc, brow, (k0 + bkof) * es)) : z;
    uint32_t af[4];
    ldsm_x4(af, aaddr);
    if constexpr (NT == 2) {
      uint32_t bf[4];
      ldsm_x4(bf, baddr);
      MmaKind<T>::mma(c[0], af, bf[0], bf[1]);
      MmaKind<T>::mma(c[NT - 1], af, bf[2], bf[3]);
    } else {
      uint32_t b0f, b1f;
      ldsm_x2(b0f, b1f, baddr);  // lanes 0-15 give the addresses
      MmaKind<T>::mma(c[0], af, b0f, b1f);
    }
  }
}

// The accumulators of an R x C Gram (R <= 16, C <= 16) into a row-major
// R x C array in shared memory; c[t][0..1] hold row lane / 4, c[t][2..3] row
// lane / 4 + 8, at columns 8 t + 2 (lane % 4) + {0, 1}.
template <int R, int C>
__device__ __forceinline__ void gram_mma_store(float* gram, const float (&c)[(C + 7) / 8][4], int lane) {
  constexpr int NT = (C + 7) / 8;
  const int r = lane >> 2;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int col = 8 * t + 2 * (lane & 3);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = r + 8 * h;
#pragma unroll
      for (int e = 0; e < 2; ++e)
        if (row < R && col + e < C) gram[row * C + col + e] = c[t][2 * h + e];
    }
  }
  __syncwarp();
}

// The token's parameter gradients from its Gram, then the Gram cleared for
// the warp's next token. With the projection the extra sums are linear in
// the plain Gram M = G X^T: rho_i = sum_d g_i v^T x = sum_j v_j M_ij and
// bp_j = sum_d (c^T g) x_j = sum_i c_i M_ij, so grad_Phi_ij = M_ij - v_j rho_i
// and grad_v_j = rho_j - sum_i Phi_ij rho_i + bp_j (reference
// ops/stream_mix_small_nb.py:379-384). Register arrays are indexed with
// constants only (selects over the runtime row and column).
template <typename P, int N, bool FUSED, bool PROJ>
__device__ __forceinline__ void bwd_gram_finish(const MixBwdArgs& a, const TokParams<P, N, FUSED, PROJ>& pr,
                                                float* gram, int64_t t, int lane) {
  using G = GramShape<N, FUSED>;
  constexpr int NA = G::NA;
  __syncwarp();
  float rho[PROJ ? N : 1];
  if constexpr (PROJ) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float r = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) r = fmaf(pr.vv[j], gram[i * NA + j], r);
      rho[i] = r;
    }
  }
  if (a.grad_phi) {
#pragma unroll
    for (int q = 0; q < (N * N + 31) / 32; ++q) {
      const int k = lane + 32 * q;
      if (k < N * N) {
        const int i = k / N, j = k % N;
        float s = gram[i * NA + j];
        if constexpr (PROJ) {
          float vj = 0.f, ri = 0.f;
#pragma unroll
          for (int q2 = 0; q2 < N; ++q2) {
            vj = q2 == j ? pr.vv[q2] : vj;
            ri = q2 == i ? rho[q2] : ri;
          }
          s = fmaf(-vj, ri, s);
        }
        a.grad_phi[t * (N * N) + k] = s;
      }
    }
  }
  if constexpr (PROJ) {
    if (a.grad_v != nullptr && lane < N) {
      const int j = lane;
      float ptr = 0.f, bp = 0.f, rj = 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float pij = 0.f;
#pragma unroll
        for (int jj = 0; jj < N; ++jj) pij = jj == j ? pr.phi[i * N + jj] : pij;
        ptr = fmaf(pij, rho[i], ptr);
        bp = fmaf(pr.cc[i], gram[i * NA + j], bp);
        rj = i == j ? rho[i] : rj;
      }
      a.grad_v[t * N + j] = (rj - ptr) + bp;
    }
  }
  if constexpr (FUSED) {
    if (lane < N) {
      if (a.grad_alpha) a.grad_alpha[t * N + lane] = gram[N * NA + lane];
      if (a.grad_beta) a.grad_beta[t * N + lane] = gram[lane * NA + N];
    }
  }
  __syncwarp();
  for (int k = lane; k < G::SIZE; k += 32) gram[k] = 0.f;
  __syncwarp();
}

template <typename T, typename P, int N, bool FUSED, bool PROJ, int W, bool BLK, bool MMA, bool SWZ>
__global__ void __launch_bounds__(bwd_warp_cap(N, BLK) * 32, 1)
mix_bwd_warp_kernel(const MixBwdArgs a, const WarpGeometry geo, const __grid_constant__ RingMaps maps) {
  static_assert(!MMA || (BLK && sizeof(T) == 2), "the tensor-core Gram is a blocked, half-precision path");
  static_assert(!SWZ || MMA, "swizzled stages belong to the tensor-core Gram");
  using L = BwdLayout<N, FUSED, PROJ>;
  constexpr int NIN = FUSED ? 4 : 2;
  constexpr int es = sizeof(T);
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // the swizzled stages of the tensor-core path start on a 1024-byte boundary
  // (geo.smem_bytes holds kSwzAlign bytes of slack for it)
  uint8_t* const smem = SWZ ? smem_raw + ((kSwzAlign - (smem_u32(smem_raw) & (kSwzAlign - 1))) & (kSwzAlign - 1))
                            : smem_raw;
  __shared__ RingState st;
  // per-consumer Gram of the blocked path
  __shared__ float gram_all[BLK ? (kWarpMaxWarps - 1) * GramShape<N, FUSED>::SIZE : 1];
  pdl_launch_dependents();
  ring_init(st, geo.stages);
  pdl_wait_prior_grid();

  const int64_t T_ = a.T, D = a.D;
  const UnitMap um = unit_map(T_, geo.tpi);
  const int nunits = um.nunits;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = geo.stages, C = geo.consumers, ns = geo.ns;
  const uint32_t rowb = static_cast<uint32_t>(geo.pitch) * es;
  const uint32_t nreg = static_cast<uint32_t>(geo.tpi) * N * rowb;  // bytes of n rows x tpi tokens
  const uint32_t oreg = static_cast<uint32_t>(geo.tpi) * rowb;      // bytes of 1 row x tpi tokens
  const bool single = geo.tpi == 1;

  if (warp == 0) {
    if (lane < geo.producers) {
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
      if (FUSED && geo.side) {
        ring_produce<T, 2>(st, geo, smem, D, um, base, rows, lane, &maps);
      } else {
        ring_produce<T, NIN>(st, geo, smem, D, um, base, rows, lane, &maps);
      }
    }
  } else if (warp - 1 < C) {
    const int c = warp - 1;
    constexpr bool PAIRS = use_pairs(N) && !BLK;  // the blocked path keeps scalar parameters
    constexpr bool BLOCKED = BLK;
    using Params = std::conditional_t<PAIRS, TokParams2<P, N, FUSED, PROJ>, TokParams<P, N, FUSED, PROJ>>;
    Params pr;
    float acc[BLOCKED ? 1 : L::kPad];
    float cg[MMA ? GramMma<N, FUSED>::NT : 1][4];  // tensor-core Gram accumulators of the token
    float2 acc2[PAIRS ? L::kAcc : 1];
    float* gram = gram_all + c * GramShape<N, FUSED>::SIZE;
    // side rows (geo.side: fused, whole tokens): two slots of this consumer
    // after the ring's stages; the next unit's rows are in flight while a
    // unit computes
    constexpr bool SIDE_OK = FUSED && PAIRS;
    const bool side = SIDE_OK && geo.side;
    const size_t side_slot_bytes = static_cast<size_t>(2) * geo.tpi * D * es;
    uint8_t* const side_base =
        smem + static_cast<size_t>(S) * geo.stage_bytes + static_cast<size_t>(c) * 2 * side_slot_bytes;
    int side_slot = 0;
    const uint8_t* side_cur = nullptr;  // the current unit's slot
    if constexpr (SIDE_OK) {
      if (side && c < nunits) side_fetch<T>(side_base, a, um.tok(c), um.cnt(c, geo.tpi), geo.tpi, lane);
    }
    if constexpr (BLOCKED) {
      for (int k = lane; k < GramShape<N, FUSED>::SIZE; k += 32) gram[k] = 0.f;
      __syncwarp();
    }
    RingCursor cur{c, 0u, c};
    for (int g0 = 0; g0 < nunits; g0 += C) {
      const int Wg = min(C, nunits - g0);
      if (c >= Wg) break;
      const int u = g0 + c;
      const int cnt = um.cnt(u, geo.tpi);
      const int64_t t0 = um.tok(u);
      pr.load(a.phi, a.v, a.alpha, a.beta, t0);  // overlaps the wait for the data
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
        auto token = [&](int tt, int64_t t) {
          if (p == 0) {
            if (tt > 0) pr.load(a.phi, a.v, a.alpha, a.beta, t);
            if constexpr (!BLOCKED) {
#pragma unroll
              for (int k = 0; k < L::kPad; ++k) acc[k] = 0.f;
            }
            if constexpr (MMA) {
#pragma unroll
              for (int k = 0; k < GramMma<N, FUSED>::NT; ++k) cg[k][0] = cg[k][1] = cg[k][2] = cg[k][3] = 0.f;
            }
            if constexpr (PAIRS) {
#pragma unroll
              for (int k = 0; k < L::kAcc; ++k) acc2[k] = make_float2(0.f, 0.f);
            }
          }
          const uint8_t* gs = sb + tt * N * rowb;
          const uint8_t* xs = sb + nreg + tt * N * rowb;
          const uint8_t* us = sb + 2 * nreg + tt * rowb;
          const uint8_t* fs = sb + 2 * nreg + oreg + tt * rowb;
          if constexpr (SIDE_OK) {
            if (side) {
              us = side_cur + tt * rowb;
              fs = side_cur + geo.tpi * rowb + tt * rowb;
            }
          }
          if constexpr (SWZ) {  // swizzled regions g, x, g_u, f (tpi == 1)
            const int rn = swz_region_bytes(N, geo.sl, es), r1 = swz_region_bytes(1, geo.sl, es);
            gs = sb;
            xs = sb + rn;
            us = sb + 2 * rn;
            fs = sb + 2 * rn + r1;
          }
          if constexpr (BLOCKED) {
            const int nc = geo.sl / kTmaChunk;
            bwd_grads_slice<T, P, N, FUSED, PROJ, W, SWZ>(a, pr, gs, us, geo.pitch, t, d0, len, lane, nc);
            if constexpr (MMA) {
              constexpr int X = FUSED ? 1 : 0;  // the g_u row of A and the f row of B
              gram_mma_slice<T, N, X, N, X, SWZ>(cg, gs, us, xs, fs, reinterpret_cast<const uint8_t*>(st.zrow), rowb,
                                                 nc, len, lane);
              if (p == ns - 1) {
                gram_mma_store<N + X, N + X>(gram, cg, lane);
                bwd_gram_finish<P, N, FUSED, PROJ>(a, pr, gram, t, lane);
              }
            } else {
              bwd_gram_slice<T, N, FUSED, W, 0>(gram, gs, xs, us, fs, geo.pitch, len, lane);
              if (p == ns - 1) bwd_gram_finish<P, N, FUSED, PROJ>(a, pr, gram, t, lane);
            }
          } else {
            if constexpr (PAIRS) {
              bwd_slice2<T, P, N, FUSED, PROJ, W>(a, pr, acc2, gs, xs, us, fs, geo.pitch, t, d0, len, lane);
            } else {
              bwd_slice<T, P, N, FUSED, PROJ, W>(a, pr, acc, gs, xs, us, fs, geo.pitch, t, d0, len, lane);
            }
            if (p == ns - 1) {  // token complete (tpi > 1 only with ns == 1)
              if constexpr (PAIRS) {
#pragma unroll
                for (int k = 0; k < L::kAcc; ++k) acc[k] = acc2[k].x + acc2[k].y;
              }
              bwd_finish<P, N, FUSED, PROJ>(a, pr, acc, t, lane);
            }
          }
        };
        if constexpr (SIDE_OK) {
          if (side) {  // this unit's side rows landed in its slot; start the next unit's
            side_cur = side_base + side_slot * side_slot_bytes;
            if (u + C < nunits) {
              side_fetch<T>(side_base + (side_slot ^ 1) * side_slot_bytes, a, um.tok(u + C), um.cnt(u + C, geo.tpi),
                            geo.tpi, lane);
              asm volatile("cp.async.wait_group 1;" ::: "memory");
            } else {
              asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            __syncwarp();
            side_slot ^= 1;
          }
        }
        if (single) {
          token(0, t0);
        } else {
          for (int tt = 0; tt < cnt; ++tt) token(tt, t0 + tt);
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

// ================================================================= host side
inline int warp_rows(bool bwd, bool fused, int n) {
  if (!bwd) return fused ? n + 1 : 2 * n;
  return fused ? 2 * n + 2 : 2 * n;
}

// Geometry of the ring; false when the shape does not fit it.
// Requires D % (16 / esize) == 0 and 16-byte aligned stream bases.
//   * a token whose rows exceed max_stage is cut into slices (one bulk copy
//     per row slice);
//   * tokens smaller than the item target are grouped, tpi per item, so that
//     one bulk copy per tensor moves several tokens.
// Stages, consumers and shared memory of the ring for geo.stage_bytes; false
// when fewer than 3 stages (or no consumer) fit.
// budget: bytes of stages (200 KB; a 216 KB ring measured no faster for the
// rings other than the tensor-core Gram's, which take kGramBudget)
inline bool ring_stage(WarpGeometry& geo, int warp_cap_, int64_t T, int num_sms, int slack_bytes = 0,
                       int budget = 200 * 1024) {
  const MixTuning tune = mix_tuning();
  int stages = std::min<int>(kRingMaxStages, budget / geo.stage_bytes);
  if (tune.stages > 0) stages = std::min(stages, tune.stages);
  int consumers = std::min(warp_cap_ - 1, stages - 2);
  if (tune.warps > 0) consumers = std::min(consumers, tune.warps);
  if (consumers < 1 || stages < 3) return false;
  geo.stages = stages;
  geo.consumers = consumers;
  geo.producers = 1;
  geo.side = 0;
  geo.smem_bytes = stages * geo.stage_bytes + slack_bytes;
  geo.grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms, T)));
  return true;
}

inline bool ring_geometry(WarpGeometry& geo, int rows, int warp_cap_, int64_t T, int64_t D, int esize,
                          int num_sms, bool bwd, int64_t item_bytes = 0) {
  if (T <= 0 || D <= 0 || D % (16 / esize) != 0) return false;
  const MixTuning tune = mix_tuning();
  const int64_t max_stage = 24 * 1024;
  // items of several small tokens: one bulk copy has a fixed cost, so small
  // items cap the copy rate (15 KB forward, 16 KB backward measured best; the
  // forward at n = 4, D = 768 takes two 7.5 KB tokens per item: 51.6 against
  // 55.2 us with one)
  const int64_t item_target =
      tune.stage_bytes > 0 ? tune.stage_bytes : item_bytes > 0 ? item_bytes : (bwd ? 16 : 15) * 1024;
  const int64_t tok_bytes = static_cast<int64_t>(rows) * D * esize;
  int64_t sl = D;
  int tpi = 1;
  if (tok_bytes > max_stage) {
    // a token wider than a stage: the fewest slices of at most the target
    // each (24 KB unless tuned), split evenly in multiples of 64 elements.
    // Measured on B200 against slices of a fixed ~16 KB, whose last slice is
    // a short remainder (n = 8, D = 1024: 448 + 448 + 128 elements, against
    // 2 x 512): backward +29% there, +18-19% at D = 2048, 4096, +9% at n = 6,
    // D = 4096; mix-write backward (n = 8, m = 4, D = 1024) +26%.
    const int64_t target = tune.stage_bytes > 0 ? std::min<int64_t>(tune.stage_bytes, max_stage) : max_stage;
    const int64_t ns = (tok_bytes + target - 1) / target;
    sl = ((D + ns - 1) / ns + 63) / 64 * 64;
    if (sl >= D) sl = D;
  } else if (tok_bytes < item_target) {
    // the fused and stream-mixing rings take the token count nearest their
    // target, within a stage; measured on B200 against rounding down: forward
    // 57.1 -> 44.9 us at n = 3, D = 1024 (two 8 KB tokens an item instead of
    // one), -4 to -6% at n = 2, 3, 8 with D = 512, 1024; backward 39.8 ->
    // 36.5 us at n = 2, D = 512; steps within 0.4% elsewhere. The read rings
    // (explicit item target) and the tuning hook round down (the read
    // backward at n = 4, m = 1, D = 768 is 7% slower with 22.5 KB items).
    const bool nearest = tune.stage_bytes <= 0 && item_bytes <= 0;
    tpi = static_cast<int>(std::min<int64_t>(
        8, std::max<int64_t>(1, (item_target + (nearest ? tok_bytes / 2 : 0)) / tok_bytes)));
    while (tpi > 1 && tpi * tok_bytes > max_stage) --tpi;
  }
  geo.tpi = tpi;
  geo.sl = static_cast<int>(sl);
  geo.ns = static_cast<int>((D + sl - 1) / sl);
  geo.pitch = geo.sl;
  geo.stage_bytes = static_cast<int>(tpi * rows * geo.pitch * esize);
  if (!ring_stage(geo, warp_cap_, T, num_sms)) return false;
  geo.wait_limit = wait_poll_limit();
  geo.status = nullptr;  // set by the launcher, which knows the stream
  geo.tma = 0;           // set by the launcher once it has the tensor maps
  geo.gram_mma = 0;
  return true;
}

// Backward kernels with up to 12 warps: fewer consumers than the register
// budget allows keep more stages loading (a consumer holds its stage while it
// computes). Measured best on B200 over D in 512..4096: 7 for sliced tokens;
// for whole tokens 8 at n <= 4 and all 11 at n = 5, 6.
inline void prefer_bwd_consumers(WarpGeometry& geo, int n) {
  if (mix_tuning().warps > 0) return;
  if (geo.ns > 1) {
    geo.consumers = std::min(geo.consumers, 7);
  } else if (n <= 4) {
    geo.consumers = std::min(geo.consumers, 8);
  }
}

#ifndef HC_BWD_SIDE
#define HC_BWD_SIDE 1  // build flag: the fused backward's g_u / f rows by consumer cp.async (side_fetch)
#endif
// Dynamic shared memory of a side-row backward (stages + consumer slots;
// the kernel's static shared memory comes on top, within the 227 KB limit).
constexpr int kSideSmemBudget = 220 * 1024;

// Producer lanes of the backward rings: four where a fill is small or made of
// many row copies (a token cut into slices, one copy per row slice; measured
// on B200, +6-19% for such rings and +12% for the mix-write forward), two for
// rings of whole tokens of 12 KB or more (the fused backward at n = 4,
// D = 768: 70.7 against 72.9 us with one lane and 72.0 with four).
constexpr int kSmallFillBytes = 12 * 1024;
constexpr int kManyFillLanes = 4;
constexpr int kLargeFillLanes = 2;
inline void prefer_producers(WarpGeometry& geo) {
  const int fixed = mix_tuning().producers;
  if (fixed > 0) {
    geo.producers = std::min(fixed, geo.stages);
  } else if (geo.ns > 1 || geo.stage_bytes < kSmallFillBytes) {
    geo.producers = std::min(kManyFillLanes, geo.stages);
  } else {
    geo.producers = std::min(kLargeFillLanes, geo.stages);
  }
}

// max_gram: the tensor-core Gram stages allowed (kGramSwizzled: either;
// kGramPadded: padded rows only, the launcher's fallback when the swizzled
// tensor maps cannot be encoded).
inline bool warp_geometry(WarpGeometry& geo, bool bwd, bool fused, bool proj, int n, int64_t T, int64_t D,
                          int esize, int num_sms, int max_gram = kGramSwizzled) {
  const int rows = warp_rows(bwd, fused, n);
  if (!ring_geometry(geo, rows, warp_cap(bwd, n), T, D, esize, num_sms, bwd)) return false;
  // whole tokens, one a stage, at n = 6 and 8: the blocked path on swizzled
  // stages of at most 24 KB. Measured on B200 (fused backward, bf16, 16,384
  // tokens) against the single pass: n = 8, D = 512 89.7 against 116.0 us;
  // n = 6, D = 384 / 512 / 640 / 768: 61.9 / 69.2 / 85.3 / 97.1 against
  // 64.5 / 82.6 / 98.5 / 109.6 us. Larger stages leave too few consumers
  // (n = 8, D = 640, 26.6 KB: 160.7 against 146.3 us); at n = 4 the single
  // pass stays faster (D = 768: 70.9 against 74.0 us).
  constexpr int kWholeMmaMaxStage = 24 * 1024;
  const bool whole = geo.ns == 1 && geo.tpi == 1 && n >= 6;
  if (bwd && gram_mma_dtype(esize) && ((geo.ns > 1 && bwd_blocked(n, proj, geo.ns)) || whole)) {
    // The tensor-core Gram (gram_mma_slice), on swizzled stages for even n
    // and on padded rows for odd n (measured). The swizzled rings take
    // kGramBudget of stages, sliced so that 9 stages fit: 7 consumers each
    // holding one and two loading (n = 6, D = 4096: 503 against 571 us with 8
    // stages of 24.5 KB; n = 8, D = 2048 with 22 KB instead of 26 KB stages:
    // 358 against 456 us; n = 8, D = 4096: 697 against 890 us).
    const WarpGeometry plain = geo;
    const MixTuning tune = mix_tuning();
    int cap = kGramBudget / 9;
    if (tune.stage_bytes > 0) cap = std::min(cap, static_cast<int>(tune.stage_bytes));
    bool ok = false;
    if (max_gram >= kGramSwizzled && n % 2 == 0 && D % kTmaChunk == 0 && T * n < (int64_t(1) << 31)) {
      const auto stage_of = [&](int nc) {
        return 2 * swz_region_bytes(n, nc * kTmaChunk, esize) +
               (fused ? 2 * swz_region_bytes(1, nc * kTmaChunk, esize) : 0);
      };
      const int64_t chunks = D / kTmaChunk;
      int nc;
      if (plain.ns == 1) {  // the whole token: its chunks, odd (the box's last one zero-filled)
        nc = static_cast<int>(chunks) | 1;
      } else {  // an odd number of 128-byte lines a row, as evenly split as that allows
        int nc_max = 1;
        for (int c2 = 3; c2 <= 255 && stage_of(c2) <= cap; c2 += 2) nc_max = c2;
        const int64_t ns = (chunks + nc_max - 1) / nc_max;
        nc = static_cast<int>((chunks + ns - 1) / ns) | 1;
      }
      geo.sl = nc * kTmaChunk;
      geo.pitch = geo.sl;
      geo.ns = static_cast<int>((D + geo.sl - 1) / geo.sl);
      geo.stage_bytes = stage_of(nc);
      geo.gram_mma = kGramSwizzled;
      ok = (plain.ns > 1 ? geo.ns > 1 : geo.stage_bytes <= kWholeMmaMaxStage) &&
           ring_stage(geo, warp_cap(bwd, n), T, num_sms, kSwzAlign, kGramBudget);
    }
    if (!ok && max_gram >= kGramPadded && plain.ns > 1) {
      // padded rows: the plain ring's slices, copied row by row (re-sliced
      // for 9 stages of a 216 KB ring, n = 7, D = 1536 measured 289 against
      // 250 us, and n = 5, D = 2048 242 against 231 us)
      geo = plain;
      geo.pitch = geo.sl + kGramPad;
      geo.stage_bytes = rows * geo.pitch * esize;
      geo.gram_mma = kGramPadded;
      ok = ring_stage(geo, warp_cap(bwd, n), T, num_sms);
    }
    if (!ok) geo = plain;
  }
  if (bwd) {
    const int cap = bwd_warp_cap(n, bwd_blocked(n, proj, geo.ns) || geo.gram_mma);
    geo.consumers = std::min(geo.consumers, cap - 1);
    if (cap > 8) prefer_bwd_consumers(geo, n);
    prefer_producers(geo);
    if (fused && use_pairs(n) && n % 2 == 0 && geo.ns == 1 && geo.tpi == 1 && !geo.gram_mma && HC_BWD_SIDE) {
      // side rows (side_fetch): stages of the 2n rows of g and x, then two
      // slots of g_u / f rows per consumer; consumers trimmed (at most two)
      // where the slots would leave fewer than consumers + 2 stages.
      // Measured on B200 (16,384 tokens, bf16, fused backward) against the
      // plain ring: n = 4, D = 768 75.7 -> 67.6 us; n = 2, D = 1024 69.8 ->
      // 56.8 us; n = 4, D = 1024 (7 consumers) 90.3 -> 87.1 us. Not taken
      // where it measured slower: n = 3, D = 1024 (71.7 -> 74.2 us) and
      // items of several tokens (n = 4, D = 512: 53.3 -> 55.4 us; n = 1,
      // D = 1024: 41.0 -> 42.9 us; level at n = 2, 3, D = 512).
      WarpGeometry sg = geo;
      const int slot2 = 4 * sg.tpi * static_cast<int>(D) * esize;  // a consumer's two slots
      sg.stage_bytes = 2 * n * sg.tpi * sg.pitch * esize;
      const int fit = (kSideSmemBudget - 2 * sg.stage_bytes) / (slot2 + sg.stage_bytes);
      const int consumers = std::min(sg.consumers, fit);
      int stages = consumers > 0 ? std::min(kRingMaxStages, (kSideSmemBudget - consumers * slot2) / sg.stage_bytes) : 0;
      if (mix_tuning().stages > 0) stages = std::min(stages, mix_tuning().stages);
      if (consumers >= 1 && consumers >= sg.consumers - 2 && stages >= consumers + 2) {
        sg.consumers = consumers;
        sg.stages = stages;
        sg.smem_bytes = stages * sg.stage_bytes + consumers * slot2;
        sg.side = 1;
        prefer_producers(sg);
        geo = sg;
      }
    }
  } else if (mix_tuning().producers > 0) {
    geo.producers = std::min(mix_tuning().producers, geo.stages);
  }
  return true;
}

#ifndef HC_PDL
#define HC_PDL 1  // build flag: launch the ring kernels with programmatic stream serialization
#endif

// Launch of a ring kernel (see pdl_launch_dependents).
template <typename... KArgs, typename... Args>
inline int launch_ring(void (*kernel)(KArgs...), int grid, dim3 block, int smem_bytes, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = HC_PDL;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) != cudaSuccess) {
    cudaGetLastError();
    return HC_ERR_LAUNCH;
  }
  return HC_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda); nullptr when the driver does not provide it.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Tensor maps for a ring whose tokens are cut into slices: tensor k is viewed
// as [T * rows[k]][D / 64][64] elements, box [rows[k]][sl / 64][64]. Sets
// geo.tma when every map is encoded; otherwise the ring keeps one copy per
// row. Needs D % 64 == 0, 16-byte aligned bases (the ring already does) and
// row coordinates within int32.
#ifndef HC_TMA
#define HC_TMA 1  // build flag: 0 copies every slice row by row (measurements)
#endif
inline void ring_tensor_maps(WarpGeometry& geo, RingMaps& maps, const void* const* base, const int* rows, int nin,
                             int64_t T, int64_t D, int esize) {
  geo.tma = 0;
  if (!HC_TMA || geo.ns <= 1 || geo.pitch != geo.sl || D % kTmaChunk != 0 || geo.sl % kTmaChunk != 0 || nin > 4)
    return;
  const auto encode = tensor_map_encoder();
  if (!encode) return;
  const CUtensorMapDataType dt = esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  for (int k = 0; k < nin; ++k) {
    if (T * rows[k] >= (int64_t(1) << 31)) return;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kTmaChunk), static_cast<cuuint64_t>(D / kTmaChunk),
                                static_cast<cuuint64_t>(T * rows[k])};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kTmaChunk) * esize, static_cast<cuuint64_t>(D) * esize};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTmaChunk), static_cast<cuuint32_t>(geo.sl / kTmaChunk),
                               static_cast<cuuint32_t>(rows[k])};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode(&maps.m[k], dt, 3, const_cast<void*>(base[k]), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return;
  }
  geo.tma = 1;
}

// Tensor maps of the swizzled tensor-core Gram stages (kGramSwizzled): the
// plain ring's view [T * rows[k]][D / 64][64] and box [rows[k]][sl / 64][64],
// with the 128-byte swizzle; a slice lands in the tensor's 1024-byte aligned
// region (gram_mma_slice). False when a map cannot be encoded.
inline bool ring_tensor_maps_swz(const WarpGeometry& geo, RingMaps& maps, const void* const* base, const int* rows,
                                 int nin, int64_t T, int64_t D, int esize) {
  if (esize != 2 || D % kTmaChunk != 0 || geo.sl % kTmaChunk != 0 || nin > 4) return false;
  const auto encode = tensor_map_encoder();
  if (!encode) return false;
  for (int k = 0; k < nin; ++k) {
    if (T * rows[k] >= (int64_t(1) << 31)) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kTmaChunk), static_cast<cuuint64_t>(D / kTmaChunk),
                                static_cast<cuuint64_t>(T * rows[k])};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kTmaChunk) * esize, static_cast<cuuint64_t>(D) * esize};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTmaChunk), static_cast<cuuint32_t>(geo.sl / kTmaChunk),
                               static_cast<cuuint32_t>(rows[k])};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode(&maps.m[k], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base[k]), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  return true;
}

template <typename KernelT>
inline int warp_prepare(KernelT* kernel, int smem_bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
    return HC_ERR_LAUNCH;
  return HC_OK;
}

// 32-bit words per lane access: 16-byte accesses for the forward at n <= 4,
// 8-byte accesses elsewhere; 4-byte accesses for the backward at n = 5, 6,
// which then fits 12 warps without spilling (register budget).
constexpr int fwd_lane_words(int n) { return n <= 4 ? 4 : 2; }
constexpr int bwd_lane_words(int n, bool blocked) { return blocked || n == 5 || n == 6 ? 1 : 2; }

template <typename T, typename P, bool FUSED, bool PROJ>
int launch_mix_fwd_warp(int n, const WarpGeometry& geo_in, const MixFwdArgs& a, cudaStream_t s) {
  WarpGeometry geo = geo_in;
  geo.status = timeout_word(s);
  // The forward copies slices row by row: TMA tensor copies measured no
  // faster on B200 (n = 4, 6, 8, D = 1024..2048, within 1-2%).
  RingMaps maps{};
  geo.tma = 0;
  const dim3 block((geo.consumers + 1) * 32, 1, 1);
  switch (n) {
#define HC_CASE(NN)                                                     \
  case NN: {                                                            \
    auto* k = mix_fwd_warp_kernel<T, P, NN, FUSED, PROJ, fwd_lane_words(NN)>;       \
    if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;            \
    if (int rc = launch_ring(k, geo.grid, block, geo.smem_bytes, s, a, geo, maps)) return rc; \
    break;                                                              \
  }
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

template <typename T, typename P, int N, bool FUSED, bool PROJ, bool BLK, bool MMA = false, bool SWZ = false>
int launch_bwd_kernel(const WarpGeometry& geo, const RingMaps& maps, dim3 block, const MixBwdArgs& a,
                      cudaStream_t s) {
  // the tensor-core path reads 8 bytes a lane in pass A (its Gram needs no
  // registers of sums)
  auto* k = mix_bwd_warp_kernel<T, P, N, FUSED, PROJ, MMA ? 2 : bwd_lane_words(N, BLK), BLK, MMA, SWZ>;
  if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;
  return launch_ring(k, geo.grid, block, geo.smem_bytes, s, a, geo, maps);
}

// The blocked kernel, with its Gram on the tensor cores when the geometry
// padded the ring's rows for it (half-precision streams cut into slices).
template <typename T, typename P, int N, bool FUSED, bool PROJ>
int launch_bwd_blocked(const WarpGeometry& geo, const RingMaps& maps, dim3 block, const MixBwdArgs& a,
                       cudaStream_t s) {
  if constexpr (gram_mma_dtype(sizeof(T))) {
    if constexpr (N % 2 == 0) {  // the geometry takes swizzled stages for even n only
      if (geo.gram_mma == kGramSwizzled)
        return launch_bwd_kernel<T, P, N, FUSED, PROJ, true, true, true>(geo, maps, block, a, s);
    }
    if (geo.gram_mma == kGramPadded) return launch_bwd_kernel<T, P, N, FUSED, PROJ, true, true>(geo, maps, block, a, s);
  }
  if (geo.gram_mma) return HC_ERR_LAUNCH;  // not reached: only half-precision rings take the tensor-core Gram
  return launch_bwd_kernel<T, P, N, FUSED, PROJ, true>(geo, maps, block, a, s);
}

template <typename T, typename P, int N, bool FUSED, bool PROJ>
int launch_bwd_one(const WarpGeometry& geo, const RingMaps& maps, dim3 block, const MixBwdArgs& a, cudaStream_t s) {
  if constexpr (bwd_blocked_n(N) && PROJ) {
    return launch_bwd_blocked<T, P, N, FUSED, PROJ>(geo, maps, block, a, s);
  } else {
    if constexpr (bwd_blocked_n(N)) {
      if (geo.ns > 1 || geo.gram_mma) return launch_bwd_blocked<T, P, N, FUSED, PROJ>(geo, maps, block, a, s);
    }
    return launch_bwd_kernel<T, P, N, FUSED, PROJ, false>(geo, maps, block, a, s);
  }
}

template <typename T, typename P, bool FUSED, bool PROJ>
int launch_mix_bwd_warp(int n, const WarpGeometry& geo_in, const MixBwdArgs& a, cudaStream_t s) {
  WarpGeometry geo = geo_in;
  RingMaps maps{};
  {
    const void* base[4] = {a.g, a.x, a.gu, a.f};
    const int rows[4] = {n, n, 1, 1};
    if (geo.gram_mma == kGramSwizzled) {
      if (ring_tensor_maps_swz(geo, maps, base, rows, FUSED ? 4 : 2, a.T, a.D, sizeof(T))) {
        geo.tma = 1;
      } else if (!warp_geometry(geo, true, FUSED, PROJ, n, a.T, a.D, sizeof(T), sm_count(), kGramPadded)) {
        return HC_ERR_LAUNCH;  // no swizzled maps: padded rows copied one by one
      }
    }
    // Plain TMA slices only for the blocked backward with the CUDA-core Gram
    // (fp32 streams): measured on B200, +7-11% there (n = 6, 8, D = 1024),
    // but 7-9% slower than row copies for the single pass (n = 4, D = 2048).
    if (geo.gram_mma == 0 && geo.ns > 1 && bwd_blocked(n, PROJ, geo.ns))
      ring_tensor_maps(geo, maps, base, rows, FUSED ? 4 : 2, a.T, a.D, sizeof(T));
  }
  geo.status = timeout_word(s);
  const dim3 block((geo.consumers + 1) * 32, 1, 1);
  switch (n) {
#define HC_CASE(NN)                                                     \
  case NN: {                                                            \
    if (int rc = launch_bwd_one<T, P, NN, FUSED, PROJ>(geo, maps, block, a, s)) return rc; \
    break;                                                              \
  }
    HC_CASE(1) HC_CASE(2) HC_CASE(3) HC_CASE(4) HC_CASE(5) HC_CASE(6) HC_CASE(7) HC_CASE(8)
#undef HC_CASE
    default: return HC_ERR_UNSUPPORTED_N;
  }
  return launch_status();
}

// Per-dtype entry points of the ring kernels (mix_*.cu).
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
