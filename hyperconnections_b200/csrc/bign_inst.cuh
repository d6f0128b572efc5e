// bign_inst.cuh — instantiates the n > 8 stream_mix_add kernels for one stream
// dtype. Included by bign_<dtype>.cu with HC_T, HC_SUFFIX and HC_T_IS_F32.
#include "bign_ring.cuh"

#define HC_CAT2(a, b) a##b
#define HC_CAT(a, b) HC_CAT2(a, b)

namespace hc {
namespace {
// Half-precision streams with D a multiple of 64 and aligned rows take the
// ring kernels on the tensor cores (bign_ring.cuh); every other shape the
// one-CTA-per-token kernels (bign.cuh).
template <typename T, typename P>
int big_fwd_p(bool proj, bool vec, int n, const MixFwdArgs& a, cudaStream_t s) {
  const int rc = proj ? launch_big_fwd_ring<T, P, true>(n, a, s) : launch_big_fwd_ring<T, P, false>(n, a, s);
  if (rc != HC_ERR_UNSUPPORTED_N) return rc;
  if (proj) return vec ? launch_big_fwd<T, P, true, true>(n, a, s) : launch_big_fwd<T, P, true, false>(n, a, s);
  return vec ? launch_big_fwd<T, P, false, true>(n, a, s) : launch_big_fwd<T, P, false, false>(n, a, s);
}
template <typename T, typename P>
int big_bwd_p(bool proj, int n, const MixBwdArgs& a, cudaStream_t s) {
  const int rc = proj ? launch_big_bwd_ring<T, P, true>(n, a, s) : launch_big_bwd_ring<T, P, false>(n, a, s);
  if (rc != HC_ERR_UNSUPPORTED_N) return rc;
  return proj ? launch_big_bwd<T, P, true, false>(n, a, s) : launch_big_bwd<T, P, false, false>(n, a, s);
}
}  // namespace

int HC_CAT(big_fwd_, HC_SUFFIX)(bool proj, bool vec, bool param_is_f32, int n, const MixFwdArgs& a,
                               cudaStream_t s) {
  using T = HC_T;
#if HC_T_IS_F32
  (void)param_is_f32;
  return big_fwd_p<T, float>(proj, vec, n, a, s);
#else
  return param_is_f32 ? big_fwd_p<T, float>(proj, vec, n, a, s) : big_fwd_p<T, T>(proj, vec, n, a, s);
#endif
}

// The backward stages the token through shared memory with element loads;
// `vec` does not change it.
int HC_CAT(big_bwd_, HC_SUFFIX)(bool proj, bool vec, bool param_is_f32, int n, const MixBwdArgs& a,
                               cudaStream_t s) {
  using T = HC_T;
  (void)vec;
#if HC_T_IS_F32
  (void)param_is_f32;
  return big_bwd_p<T, float>(proj, n, a, s);
#else
  return param_is_f32 ? big_bwd_p<T, float>(proj, n, a, s) : big_bwd_p<T, T>(proj, n, a, s);
#endif
}
}  // namespace hc
