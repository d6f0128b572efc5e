// generator.cu — CGHC's generator A per token (n <= 8), forward and backward,
// as kernels of one thread per token over generator.cuh.
#include "generator.cuh"

namespace hc {
namespace {

template <int N, bool VEC>
__global__ void __launch_bounds__(kGenThreads) gen_fwd_kernel(const GenArgs a, int flags) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= a.T) return;
  float A[N * N];
  gen_forward_token<N, VEC>(a, flags, t, A);
#pragma unroll
  for (int k = 0; k < N * N; ++k) a.A[t * N * N + k] = A[k];
}

template <int N, bool VEC>
__global__ void __launch_bounds__(kGenThreads) gen_bwd_kernel(const GenArgs a, int flags) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= a.T) return;
  float G[N * N];
#pragma unroll
  for (int k = 0; k < N * N; ++k) G[k] = a.G[t * N * N + k];
  gen_backward_token<N, VEC>(a, flags, t, G);
}

#define HC_GEN_SWITCH(n, LAUNCH) \
  switch (n) {                   \
    case 1: LAUNCH(1); break;    \
    case 2: LAUNCH(2); break;    \
    case 3: LAUNCH(3); break;    \
    case 4: LAUNCH(4); break;    \
    case 5: LAUNCH(5); break;    \
    case 6: LAUNCH(6); break;    \
    case 7: LAUNCH(7); break;    \
    case 8: LAUNCH(8); break;    \
    default: return HC_ERR_UNSUPPORTED_N; \
  }

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_cghc_generator_fwd(const float* M, const float* lc, const float* R, const float* dpre,
                                     const float* S, const float* ld, float* A, int64_t T, int n, int vec_dt,
                                     int flags, float dt_min_c, float dt_max_c, float dt_min_d, float dt_max_d,
                                     void* stream) {
  HC_ENTRY("hc_cghc_generator_fwd");
  GenArgs a{};
  a.M = M; a.lc = lc; a.ld = ld; a.R = R; a.dpre = dpre; a.S = S; a.A = A; a.T = T;
  a.lo_c = dt_min_c; a.hi_c = dt_max_c; a.lo_d = dt_min_d; a.hi_d = dt_max_d;
  int rc = check_gen(a, n, flags);
  if (rc || T == 0) return rc;
  if (!A) return HC_ERR_NULL_POINTER;
  const unsigned grid = static_cast<unsigned>((T + kGenThreads - 1) / kGenThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define L(NN)                                                                         \
  if (vec_dt) gen_fwd_kernel<NN, true><<<grid, kGenThreads, 0, st>>>(a, flags);      \
  else gen_fwd_kernel<NN, false><<<grid, kGenThreads, 0, st>>>(a, flags)
  HC_GEN_SWITCH(n, L)
#undef L
  return launch_status();
}

extern "C" int hc_cghc_generator_bwd(const float* M, const float* lc, const float* R, const float* dpre,
                                     const float* S, const float* ld, const float* G, float* dM, float* dlc,
                                     float* dR, float* ddpre, float* dS, float* dld, int64_t T, int n, int vec_dt,
                                     int flags, float dt_min_c, float dt_max_c, float dt_min_d, float dt_max_d,
                                     void* stream) {
  HC_ENTRY("hc_cghc_generator_bwd");
  GenArgs a{};
  a.M = M; a.lc = lc; a.ld = ld; a.R = R; a.dpre = dpre; a.S = S; a.G = G; a.T = T;
  a.dM = dM; a.dlc = dlc; a.dld = dld; a.dR = dR; a.ddpre = ddpre; a.dS = dS;
  a.lo_c = dt_min_c; a.hi_c = dt_max_c; a.lo_d = dt_min_d; a.hi_d = dt_max_d;
  int rc = check_gen(a, n, flags);
  if (rc || T == 0) return rc;
  if (!G) return HC_ERR_NULL_POINTER;
  const unsigned grid = static_cast<unsigned>((T + kGenThreads - 1) / kGenThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define L(NN)                                                                         \
  if (vec_dt) gen_bwd_kernel<NN, true><<<grid, kGenThreads, 0, st>>>(a, flags);      \
  else gen_bwd_kernel<NN, false><<<grid, kGenThreads, 0, st>>>(a, flags)
  HC_GEN_SWITCH(n, L)
#undef L
  return launch_status();
}
