// rw_inst.cuh — instantiates the read / mix-write kernels for one stream
// dtype and one direction. Included by rw_<dtype>_<dir>.cu with HC_T (the
// element type), HC_SUFFIX (the entry-point suffix) and HC_RW_BWD (0 forward,
// 1 backward) defined, so the six units compile in parallel.
#include "rw_warp.cuh"

#define HC_CAT2(a, b) a##b
#define HC_CAT(a, b) HC_CAT2(a, b)
#if HC_RW_BWD
#define HC_RW_ENTRY HC_CAT(rw_bwd_, HC_SUFFIX)
#define HC_RW_TAKE HC_CAT(rw_bwd_take_timeouts_, HC_SUFFIX)
#else
#define HC_RW_ENTRY HC_CAT(rw_fwd_, HC_SUFFIX)
#define HC_RW_TAKE HC_CAT(rw_fwd_take_timeouts_, HC_SUFFIX)
#endif

namespace hc {

int HC_RW_ENTRY(bool ring, bool mixw, bool proj, int n, int m, const WarpGeometry& g, const RwArgs& a,
                cudaStream_t s) {
  using T = HC_T;
  constexpr bool B = HC_RW_BWD != 0;
  if (!ring) return rw_launch_generic<T>(B, n, m, mixw, a, s);
  if (!mixw) return rw_launch_ring<T, B, false, false>(n, m, g, a, s);
  return proj ? rw_launch_ring<T, B, true, true>(n, m, g, a, s) : rw_launch_ring<T, B, true, false>(n, m, g, a, s);
}

// The ring's wait-timeout counter of this translation unit.
unsigned int HC_RW_TAKE(bool reset) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_mix_wait_timeouts, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (reset && v != 0) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_mix_wait_timeouts, &z, sizeof(z));
  }
  return v;
}

}  // namespace hc
