// ring_fill_rate.cu — how fast a shared-memory ring of 1-D bulk copies can be
// filled on B200, with consumers that release every stage as soon as it has
// landed (no compute). It measures the copy machinery the stream-mixing
// kernels are built on (csrc/mix_warp.cuh), not those kernels.
//
// Build and run (one GPU, a few seconds):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o ring_fill_rate ring_fill_rate.cu && ./ring_fill_rate
//
// Part 1: one issuing thread, one item = `copies` bulk copies of `copy_bytes`,
//         over stage counts; and two CTAs per SM.
// Part 2: who issues the fills: one thread (with and without the proxy fence
//         before a refill), P lanes of one warp in lockstep, P independent
//         producer warps each owning S/P stages, or P consumer warps.
// Every CTA reads its own contiguous part of a 2 GiB buffer; a 256 MiB write
// between launches flushes L2; the best of three timed launches is printed.
// Every wait is bounded; a wait that gives up sets a flag and the program
// exits with status 2.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <vector>

namespace {

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(c) : "memory");
}
__device__ __forceinline__ bool try_wait(uint64_t* b, uint32_t ph) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0,1,0,p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(ph)
      : "memory");
  return ok;
}
__device__ __forceinline__ bool wait(uint64_t* b, uint32_t ph) {
  for (uint32_t i = 0; i < (1u << 22); ++i)
    if (try_wait(b, ph)) return true;
  return false;
}
__device__ __forceinline__ void expect_tx(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Plain 1-D bulk copy global -> this CTA's shared memory (one destination CTA).
__device__ __forceinline__ void g2s(void* d, const void* s, uint32_t n, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   su32(d)),
               "l"(s), "r"(n), "r"(su32(b))
               : "memory");
}

__device__ unsigned g_fail;

enum Mode { kOneThread = 0, kNoFence = 1, kLockstepLanes = 2, kProducerWarps = 3, kConsumerWarps = 4 };

// One producer thread issues item k (copies x cb bytes, contiguous in global)
// into stage k mod S; consumer thread(s) wait for it and release it at once.
__global__ void ring_kernel(const uint8_t* src, int64_t items, int cb, int copies, int S, int mode, int P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[32], empty[32];
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int64_t item = (int64_t)cb * copies;
  const uint8_t* base = src + (int64_t)blockIdx.x * items * item;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto fill = [&](int64_t k, int s) {
    expect_tx(&full[s], (uint32_t)item);
    uint8_t* dst = smem + (size_t)s * item;
    for (int c = 0; c < copies; ++c) g2s(dst + (size_t)c * cb, base + k * item + (int64_t)c * cb, cb, &full[s]);
  };
  if (mode == kOneThread || mode == kNoFence || mode == kConsumerWarps) {
    if (threadIdx.x == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int64_t k = 0; k < items; ++k) {
        if (k >= S && !wait(&empty[s], ph ^ 1u)) {
          atomicAdd(&g_fail, 1u);
          break;
        }
        if (mode != kNoFence) proxy_fence();
        fill(k, s);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    } else if (warp >= 1 && lane == 0) {
      const int nc = mode == kConsumerWarps ? P : 1, c = warp - 1;
      if (c < nc) {
        int s = c % S;
        uint32_t ph = (c / S) & 1;
        for (int64_t k = c; k < items; k += nc) {
          if (!wait(&full[s], ph)) {
            atomicAdd(&g_fail, 1u);
            break;
          }
          arrive(&empty[s]);
          s += nc;
          while (s >= S) {
            s -= S;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (mode == kLockstepLanes) {  // P <= S lanes, item k0 + lane per round
    if (warp == 0 && lane < P) {
      const unsigned mask = (1u << P) - 1u;
      for (int64_t k0 = 0; k0 < items; k0 += P) {
        const int64_t k = k0 + lane;
        const int s = (int)(k % S);
        const uint32_t ph = (uint32_t)((k / S) & 1);
        bool ok = true;
        if (k < items) {
          if (k >= S) ok = wait(&empty[s], ph ^ 1u);
          if (ok) {
            proxy_fence();
            fill(k, s);
          }
        }
        if (!ok) atomicAdd(&g_fail, 1u);
        if (__any_sync(mask, !ok)) break;
      }
    } else if (threadIdx.x == 32) {
      int s = 0;
      uint32_t ph = 0;
      for (int64_t k = 0; k < items; ++k) {
        if (!wait(&full[s], ph)) {
          atomicAdd(&g_fail, 1u);
          break;
        }
        arrive(&empty[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (mode == kProducerWarps) {  // pair w: producer warp w, consumer warp P + w, stages w, w + P, ...
    const int SP = S / P;
    if (lane == 0 && warp < 2 * P) {
      const int w = warp % P;
      const bool prod = warp < P;
      int j = 0;
      uint32_t ph = 0;
      for (int64_t k = w; k < items; k += P) {
        const int s = w + P * j;
        if (prod) {
          if (k >= (int64_t)S && !wait(&empty[s], ph ^ 1u)) {
            atomicAdd(&g_fail, 1u);
            break;
          }
          proxy_fence();
          fill(k, s);
        } else {
          if (!wait(&full[s], ph)) {
            atomicAdd(&g_fail, 1u);
            break;
          }
          arrive(&empty[s]);
        }
        if (++j == SP) {
          j = 0;
          ph ^= 1u;
        }
      }
    }
  }
  __syncthreads();
}

struct Cfg {
  int cb, copies, S, ctas_per_sm, mode, P;
};

}  // namespace

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  const size_t total = (size_t)2 << 30;
  uint8_t *buf = nullptr, *flush = nullptr;
  if (cudaMalloc(&buf, total) != cudaSuccess || cudaMalloc(&flush, 256 << 20) != cudaSuccess) return 1;
  cudaMemset(buf, 1, total);
  cudaFuncSetAttribute(ring_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  std::vector<Cfg> cfgs;
  for (int cb : {512, 1536, 3072, 6144, 12288, 24576})
    for (int S : {4, 8, 16, 32})
      if ((int64_t)cb * S <= 200 * 1024) cfgs.push_back({cb, 1, S, 1, kOneThread, 1});
  for (int copies : {1, 2, 4, 8, 16}) cfgs.push_back({16384 / copies, copies, 12, 1, kOneThread, 1});
  for (int cb : {1536, 6144, 12288}) cfgs.push_back({cb, 1, std::min(32, (100 * 1024) / cb), 2, kOneThread, 1});
  for (int cb : {1536, 6144}) {
    const int S = 16;
    cfgs.push_back({cb, 1, S, 1, kOneThread, 1});
    cfgs.push_back({cb, 1, S, 1, kNoFence, 1});
    for (int P : {2, 4}) cfgs.push_back({cb, 1, S, 1, kLockstepLanes, P});
    for (int P : {2, 4, 8}) cfgs.push_back({cb, 1, S, 1, kProducerWarps, P});
    for (int P : {2, 4}) cfgs.push_back({cb, 1, S, 1, kConsumerWarps, P});
  }
  static const char* names[] = {"one thread", "one thread, no proxy fence", "lockstep lanes", "producer warps",
                                "consumer warps"};
  printf("copy_bytes copies stages ctas/SM issuer                      P    GB/s\n");
  for (const Cfg& c : cfgs) {
    const int64_t item = (int64_t)c.cb * c.copies;
    const int grid = sms * c.ctas_per_sm;
    const int64_t per_cta = (int64_t)(total / item) / grid;
    const size_t smem = (size_t)item * c.S;
    const int threads = 32 * (c.mode == kProducerWarps ? 2 * c.P : (c.mode == kConsumerWarps ? 1 + c.P : 2));
    float best = 1e30f;
    for (int rep = 0; rep < 4; ++rep) {
      cudaMemsetAsync(flush, rep, 256 << 20);
      cudaEventRecord(e0);
      ring_kernel<<<grid, threads, smem>>>(buf, per_cta, c.cb, c.copies, c.S, c.mode, c.P);
      cudaEventRecord(e1);
      cudaEventSynchronize(e1);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      if (rep > 0 && ms < best) best = ms;
    }
    const cudaError_t err = cudaGetLastError();
    unsigned fail = 0;
    cudaMemcpyFromSymbol(&fail, g_fail, sizeof(fail));
    if (err != cudaSuccess || fail) {
      printf("error %d, %u waits gave up\n", (int)err, fail);
      return 2;
    }
    printf("%10d %6d %6d %7d %-27s %2d %7.0f\n", c.cb, c.copies, c.S, c.ctas_per_sm, names[c.mode], c.P,
           (double)per_cta * grid * item / best / 1e6);
  }
  return 0;
}
