// status.cu — process-wide state of libhcops: the status word of the bounded
// waits, and the two debug knobs (ring geometry, wait poll limit).
//
// The status word lives in pinned host memory mapped into every device's
// address space (cudaHostAllocMapped | cudaHostAllocPortable; with unified
// addressing the host pointer is also the device pointer). A kernel whose wait
// gives up adds 1 to it with a system-scope atomic; the host reads it with a
// plain load, so checking it costs an entry point no synchronisation. It is
// mapped once, at the first launch of a kernel with bounded waits that is not
// being captured into a CUDA graph.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "mix_warp.cuh"

#ifndef HC_PRODUCER_LANES
#define HC_PRODUCER_LANES 0  // build flag: fixed producer lanes of every ring (0 = automatic)
#endif

namespace hc {
namespace {

std::atomic<unsigned int*> g_word{nullptr};
std::mutex g_word_mutex;

std::atomic<int> g_stage_bytes{0}, g_stages{0}, g_warps{0}, g_producers{0};
std::atomic<uint32_t> g_wait_limit{kWaitPolls};

}  // namespace

unsigned int* timeout_word(cudaStream_t s) {
  unsigned int* w = g_word.load(std::memory_order_acquire);
  if (w) return w;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cap != cudaStreamCaptureStatusNone) return nullptr;  // no allocation inside a capture
  std::lock_guard<std::mutex> lock(g_word_mutex);
  w = g_word.load(std::memory_order_acquire);
  if (w) return w;
  void* p = nullptr;
  if (cudaHostAlloc(&p, 64, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, p, 0) != cudaSuccess || d != p) {
    // no unified addressing: the host and device addresses differ, keep none
    cudaGetLastError();
    cudaFreeHost(p);
    return nullptr;
  }
  *static_cast<volatile unsigned int*>(p) = 0u;
  w = static_cast<unsigned int*>(p);
  g_word.store(w, std::memory_order_release);
  return w;
}

int pending_timeout() {
  const unsigned int* w = g_word.load(std::memory_order_acquire);
  if (w && *reinterpret_cast<const volatile unsigned int*>(w) != 0u) return HC_ERR_TIMEOUT;
  return HC_OK;
}

void clear_timeout_word() {
  unsigned int* w = g_word.load(std::memory_order_acquire);
  if (w) *reinterpret_cast<volatile unsigned int*>(w) = 0u;
}

uint32_t wait_poll_limit() { return g_wait_limit.load(std::memory_order_relaxed); }

MixTuning mix_tuning() {
  const int lanes = g_producers.load(std::memory_order_relaxed);
  return MixTuning{g_stage_bytes.load(std::memory_order_relaxed), g_stages.load(std::memory_order_relaxed),
                   g_warps.load(std::memory_order_relaxed), lanes > 0 ? lanes : HC_PRODUCER_LANES};
}

}  // namespace hc

extern "C" int hc_debug_set_mix_tuning(int stage_bytes, int stages, int warps, int producers) {
  if (stage_bytes < 0 || stages < 0 || stages > hc::kRingMaxStages || warps < 0 || warps >= hc::kWarpMaxWarps ||
      producers < 0 || producers > 32)
    return HC_ERR_BAD_SIZE;
  hc::g_stage_bytes.store(stage_bytes, std::memory_order_relaxed);
  hc::g_stages.store(stages, std::memory_order_relaxed);
  hc::g_warps.store(warps, std::memory_order_relaxed);
  hc::g_producers.store(producers, std::memory_order_relaxed);
  return HC_OK;
}

extern "C" int hc_debug_set_wait_limit(unsigned int polls) {
  hc::g_wait_limit.store(polls == 0 ? hc::kWaitPolls : polls, std::memory_order_relaxed);
  return HC_OK;
}

extern "C" int hc_timeout_status(unsigned int* count) {
  if (!count) return HC_ERR_NULL_POINTER;
  const unsigned int* w = hc::g_word.load(std::memory_order_acquire);
  *count = w ? *reinterpret_cast<const volatile unsigned int*>(w) : 0u;
  return HC_OK;
}
