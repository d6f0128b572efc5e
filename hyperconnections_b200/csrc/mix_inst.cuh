// mix_inst.cuh — instantiates the mixing kernels for one stream dtype.
// Included by mix_f32.cu / mix_f16.cu / mix_bf16.cu with HC_T (the element
// type) and HC_SUFFIX (the entry-point suffix) defined, so the three dtypes
// compile as separate translation units in parallel.
#include "mix_warp.cuh"

#define HC_CAT2(a, b) a##b
#define HC_CAT(a, b) HC_CAT2(a, b)

namespace hc {
namespace {

template <typename T, typename P>
int add_fwd(bool proj, bool vec, int n, const MixGeometry& g, const MixFwdArgs& a, cudaStream_t s) {
  if (proj)
    return vec ? launch_mix_fwd<T, P, false, true, true>(n, g, a, s)
               : launch_mix_fwd<T, P, false, true, false>(n, g, a, s);
  return vec ? launch_mix_fwd<T, P, false, false, true>(n, g, a, s)
             : launch_mix_fwd<T, P, false, false, false>(n, g, a, s);
}

template <typename T, typename P>
int add_bwd(bool proj, bool vec, int n, const MixGeometry& g, const MixBwdArgs& a, cudaStream_t s) {
  if (proj)
    return vec ? launch_mix_bwd<T, P, false, true, true>(n, g, a, s)
               : launch_mix_bwd<T, P, false, true, false>(n, g, a, s);
  return vec ? launch_mix_bwd<T, P, false, false, true>(n, g, a, s)
             : launch_mix_bwd<T, P, false, false, false>(n, g, a, s);
}

template <typename T, typename P>
int add_fwd_warp(bool proj, int n, const WarpGeometry& g, const MixFwdArgs& a, cudaStream_t s) {
  return proj ? launch_mix_fwd_warp<T, P, false, true>(n, g, a, s) : launch_mix_fwd_warp<T, P, false, false>(n, g, a, s);
}

template <typename T, typename P>
int add_bwd_warp(bool proj, int n, const WarpGeometry& g, const MixBwdArgs& a, cudaStream_t s) {
  return proj ? launch_mix_bwd_warp<T, P, false, true>(n, g, a, s) : launch_mix_bwd_warp<T, P, false, false>(n, g, a, s);
}

}  // namespace

int HC_CAT(mix_fwd_warp_, HC_SUFFIX)(bool fused, bool proj, bool param_is_f32, int n, const WarpGeometry& g,
                                   const MixFwdArgs& a, cudaStream_t s) {
  using T = HC_T;
  if (fused) return launch_mix_fwd_warp<T, float, true, false>(n, g, a, s);
#if HC_T_IS_F32
  (void)param_is_f32;
  return add_fwd_warp<T, float>(proj, n, g, a, s);
#else
  return param_is_f32 ? add_fwd_warp<T, float>(proj, n, g, a, s) : add_fwd_warp<T, T>(proj, n, g, a, s);
#endif
}

int HC_CAT(mix_bwd_warp_, HC_SUFFIX)(bool fused, bool proj, bool param_is_f32, int n, const WarpGeometry& g,
                                   const MixBwdArgs& a, cudaStream_t s) {
  using T = HC_T;
  if (fused) return launch_mix_bwd_warp<T, float, true, false>(n, g, a, s);
#if HC_T_IS_F32
  (void)param_is_f32;
  return add_bwd_warp<T, float>(proj, n, g, a, s);
#else
  return param_is_f32 ? add_bwd_warp<T, float>(proj, n, g, a, s) : add_bwd_warp<T, T>(proj, n, g, a, s);
#endif
}

unsigned int HC_CAT(mix_warp_take_timeouts_, HC_SUFFIX)(bool reset) {
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

int HC_CAT(mix_fwd_, HC_SUFFIX)(bool fused, bool proj, bool vec, bool param_is_f32, int n,
                               const MixGeometry& g, const MixFwdArgs& a, cudaStream_t s) {
  using T = HC_T;
  if (fused)
    return vec ? launch_mix_fwd<T, float, true, false, true>(n, g, a, s)
               : launch_mix_fwd<T, float, true, false, false>(n, g, a, s);
#if HC_T_IS_F32
  (void)param_is_f32;
  return add_fwd<T, float>(proj, vec, n, g, a, s);
#else
  return param_is_f32 ? add_fwd<T, float>(proj, vec, n, g, a, s) : add_fwd<T, T>(proj, vec, n, g, a, s);
#endif
}

int HC_CAT(mix_bwd_, HC_SUFFIX)(bool fused, bool proj, bool vec, bool param_is_f32, int n,
                               const MixGeometry& g, const MixBwdArgs& a, cudaStream_t s) {
  using T = HC_T;
  if (fused)
    return vec ? launch_mix_bwd<T, float, true, false, true>(n, g, a, s)
               : launch_mix_bwd<T, float, true, false, false>(n, g, a, s);
#if HC_T_IS_F32
  (void)param_is_f32;
  return add_bwd<T, float>(proj, vec, n, g, a, s);
#else
  return param_is_f32 ? add_bwd<T, float>(proj, vec, n, g, a, s) : add_bwd<T, T>(proj, vec, n, g, a, s);
#endif
}

}  // namespace hc
