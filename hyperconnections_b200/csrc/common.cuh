// common.cuh — shared device helpers for the hyper-connections kernels.
//
// Stream data moves in 16-byte chunks (8 bf16/fp16 or 4 fp32 elements) with
// non-coherent, L1-bypassing loads; all arithmetic is fp32. Conversions to the
// 16-bit types round to nearest even, like the reference's tl.store into a
// bf16/fp16 tensor.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

#include "../../include/hcops.h"

namespace hc {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------- elements
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kVec = 4;
  __device__ static __forceinline__ float to_f(float v) { return v; }
  __device__ static __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__half> {
  static constexpr int kVec = 8;
  __device__ static __forceinline__ float to_f(__half v) { return __half2float(v); }
  __device__ static __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ static __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// ---------------------------------------------------------------- raw loads
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ void st_v4(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// unpack one 16-byte chunk into kVec floats
template <typename T> __device__ __forceinline__ void unpack(const uint4& v, float* f);
template <> __device__ __forceinline__ void unpack<float>(const uint4& v, float* f) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}
template <> __device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& v, float* f) {
  // bf16 -> fp32 is exact: the 16 bits become the high half of the fp32 word
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <> __device__ __forceinline__ void unpack<__half>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 p = __half22float2(h);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

template <typename T> __device__ __forceinline__ uint4 pack(const float* f);
template <> __device__ __forceinline__ uint4 pack<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                    __float_as_uint(f[2]), __float_as_uint(f[3]));
}
template <> __device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <> __device__ __forceinline__ uint4 pack<__half>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// A chunk is E consecutive elements of one stream row. VECTOR chunks are one
// 16-byte access (the host guarantees D % kVec == 0 and 16-byte aligned bases);
// scalar chunks are a single element (any D, any element alignment).
template <typename T, bool VECTOR> struct Chunk {
  static constexpr int E = VECTOR ? Elem<T>::kVec : 1;
  __device__ static __forceinline__ void load(const T* p, bool ok, float (&f)[E]) {
    if constexpr (VECTOR) {
      if (ok) {
        unpack<T>(ld_nc_v4(p), f);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) f[e] = 0.f;
      }
    } else {
      f[0] = ok ? Elem<T>::to_f(__ldg(p)) : 0.f;
    }
  }
  __device__ static __forceinline__ void store(T* p, bool ok, const float (&f)[E]) {
    if (!ok) return;
    if constexpr (VECTOR) {
      st_v4(p, pack<T>(f));
    } else {
      p[0] = Elem<T>::from_f(f[0]);
    }
  }
};

// ------------------------------------------------------- small parameter rows
// Loads that the compiler may not repeat: values a thread keeps in registers
// for a whole token (re-loading them inside the element loops would put an L1
// round trip in front of every chunk).
__device__ __forceinline__ float4 ldg_keep_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ float ldg_keep_f32(const float* p) {
  float r;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ unsigned short ldg_keep_u16(const void* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

template <typename P> __device__ __forceinline__ float ldg_keep_elem(const P* p);
template <> __device__ __forceinline__ float ldg_keep_elem<float>(const float* p) { return ldg_keep_f32(p); }
template <> __device__ __forceinline__ float ldg_keep_elem<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __uint_as_float(static_cast<uint32_t>(ldg_keep_u16(p)) << 16);
}
template <> __device__ __forceinline__ float ldg_keep_elem<__half>(const __half* p) {
  return __half2float(__ushort_as_half(ldg_keep_u16(p)));
}

// K consecutive parameters loaded once into registers (see ldg_keep_f4).
template <typename P, int K>
__device__ __forceinline__ void load_params_keep(const P* __restrict__ src, float (&dst)[K]) {
  if constexpr (sizeof(P) == 4 && (K % 4) == 0) {
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
#pragma unroll
      for (int k = 0; k < K; k += 4) {
        const float4 q = ldg_keep_f4(reinterpret_cast<const float*>(src) + k);
        dst[k] = q.x; dst[k + 1] = q.y; dst[k + 2] = q.z; dst[k + 3] = q.w;
      }
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) dst[k] = ldg_keep_elem<P>(src + k);
}
// Load K consecutive parameters (converted to fp32). Vector path when the row
// starts on a 16-byte boundary and K*4 is a multiple of 16 (fp32 params).
template <typename P, int K>
__device__ __forceinline__ void load_params(const P* __restrict__ src, float (&dst)[K]) {
  if constexpr (sizeof(P) == 4 && (K % 4) == 0) {
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
#pragma unroll
      for (int k = 0; k < K; k += 4) {
        float4 q = __ldg(reinterpret_cast<const float4*>(src) + k / 4);
        dst[k] = q.x; dst[k + 1] = q.y; dst[k + 2] = q.z; dst[k + 3] = q.w;
      }
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) dst[k] = Elem<P>::to_f(__ldg(src + k));
}

// ------------------------------------------------------ warp transpose-reduce
// v holds 32*R partial sums per lane. After the call lane l holds, in v[0..R),
// the warp-wide sums of indices [R*l, R*l + R). Costs 31*R shuffles instead of
// the 5*32*R of one butterfly per value: every step sends half of the live
// values and keeps the other half.
template <int L>
__device__ __forceinline__ void tr_step(float* v, int lane, int o) {
  constexpr int H = L / 2;
  const bool upper = (lane & o) != 0;
#pragma unroll
  for (int i = 0; i < H; ++i) {
    float send = upper ? v[i] : v[i + H];
    float keep = upper ? v[i + H] : v[i];
    v[i] = keep + __shfl_xor_sync(kFull, send, o);
  }
}

template <int R>
__device__ __forceinline__ void warp_transpose_reduce(float* v, int lane) {
  tr_step<32 * R>(v, lane, 16);
  tr_step<16 * R>(v, lane, 8);
  tr_step<8 * R>(v, lane, 4);
  tr_step<4 * R>(v, lane, 2);
  tr_step<2 * R>(v, lane, 1);
}

// --------------------------------------------------------------- host helpers
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HC_OK : HC_ERR_LAUNCH;
}

// SM count of the current device (cached per device; 148 when unknown).
inline int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev < 64) cached[dev] = n;
  return n;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

inline int dtype_size(int dt) {
  switch (dt) {
    case HC_DTYPE_F32: return 4;
    case HC_DTYPE_F16: return 2;
    case HC_DTYPE_BF16: return 2;
    default: return 0;
  }
}

// Bounded waits of the expm kernels that gave up (expm.cu); summed into
// hc_wait_timeouts() with those of the ring kernels.
unsigned int expm_take_timeouts(bool reset);

// ------------------------------------------------------ bounded-wait status
// Every spin-wait in the kernels polls at most a fixed number of times. A wait
// that gives up leaves its kernel's outputs incomplete; the kernel counts the
// event in a per-translation-unit device counter and in ONE word of pinned,
// device-mapped host memory shared by the process (status.cu). Every entry
// point that launches work reads that word first and returns HC_ERR_TIMEOUT
// while it is non-zero, until hc_wait_timeouts(..., reset = 1) clears it, so
// a caller learns of the give-up at its next call (like a sticky CUDA error).
constexpr uint32_t kWaitPolls = 1u << 22;  // default poll limit of every data wait

// Device-visible address of the status word, mapped on first use (never while
// stream s is capturing a graph); nullptr when it cannot be mapped.
unsigned int* timeout_word(cudaStream_t s);
// HC_ERR_TIMEOUT when some kernel has reported a give-up, else HC_OK; never
// maps the word (a plain host read of it when it exists).
int pending_timeout();
// Clears the status word (hc_wait_timeouts with reset).
void clear_timeout_word();
// Poll limit of the data waits: kWaitPolls unless hc_debug_set_wait_limit
// lowered it. The exit drains of the rings always use kWaitPolls.
uint32_t wait_poll_limit();

// Ring geometry overrides of hc_debug_set_mix_tuning (0 = automatic), read
// atomically at every launch.
struct MixTuning {
  int stage_bytes;  // target bytes of an item of several small tokens
  int stages;       // stages of the ring
  int warps;        // consumer warps per CTA
  int producers;    // producer lanes of warp 0
};
MixTuning mix_tuning();

__device__ __forceinline__ void report_timeout(unsigned int* counter, unsigned int* word) {
  atomicAdd(counter, 1u);
  if (word) atomicAdd_system(word, 1u);
}

// NVTX range around one C-ABI call (visible in Nsight Systems / ncu's NVTX
// filter; a no-op branch when no tool is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace hc

// First statement of every entry point that launches work: an NVTX range
// named after it, then the sticky give-up status of earlier launches.
#define HC_ENTRY(name)                  \
  const ::hc::NvtxRange hc_nvtx_(name); \
  if (const int hc_pending_ = ::hc::pending_timeout()) return hc_pending_
