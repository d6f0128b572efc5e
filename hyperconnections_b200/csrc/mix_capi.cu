// mix_capi.cu — C entry points of the stream-mixing kernels (see hcops.h).
//
// Argument checking happens here, on the host, before any launch: sizes,
// dtype codes, NULL pointers and alignment. The 16-byte vector path is taken
// when D is a multiple of the chunk width and every stream base pointer is
// 16-byte aligned; otherwise the element-wise path of the same kernels runs.
#include "bign.cuh"
#include "rw_warp.cuh"

namespace hc {
namespace {

constexpr int64_t kMaxD = int64_t(1) << 24;
constexpr int64_t kMaxTokens = (int64_t(1) << 31) - 1;

int check_dtypes(int sdt, int pdt) {
  if (dtype_size(sdt) == 0 || dtype_size(pdt) == 0) return HC_ERR_DTYPE;
  if (pdt != HC_DTYPE_F32 && pdt != sdt) return HC_ERR_DTYPE;
  return HC_OK;
}

int check_sizes(int64_t T, int n, int64_t D, int max_n = 8) {
  // one CTA row per token: the grid must stay within 2^31 - 1 CTAs
  if (T < 0 || T > kMaxTokens || D < 0 || D > kMaxD) return HC_ERR_BAD_SIZE;
  if (n < 1 || n > max_n) return HC_ERR_UNSUPPORTED_N;
  return HC_OK;
}

int run_big_fwd(int sdt, bool proj, bool vec, bool pf32, int n, const MixFwdArgs& a, cudaStream_t s) {
  switch (sdt) {
    case HC_DTYPE_F32: return big_fwd_f32(proj, vec, pf32, n, a, s);
    case HC_DTYPE_F16: return big_fwd_f16(proj, vec, pf32, n, a, s);
    case HC_DTYPE_BF16: return big_fwd_bf16(proj, vec, pf32, n, a, s);
  }
  return HC_ERR_DTYPE;
}

int run_big_bwd(int sdt, bool proj, bool pf32, int n, const MixBwdArgs& a, cudaStream_t s) {
  switch (sdt) {
    case HC_DTYPE_F32: return big_bwd_f32(proj, false, pf32, n, a, s);
    case HC_DTYPE_F16: return big_bwd_f16(proj, false, pf32, n, a, s);
    case HC_DTYPE_BF16: return big_bwd_bf16(proj, false, pf32, n, a, s);
  }
  return HC_ERR_DTYPE;
}

int vec_width(int sdt) { return sdt == HC_DTYPE_F32 ? 4 : 8; }

int run_fwd(int sdt, bool fused, bool proj, bool vec, bool pf32, int n, const MixGeometry& g,
            const MixFwdArgs& a, cudaStream_t s) {
  switch (sdt) {
    case HC_DTYPE_F32: return mix_fwd_f32(fused, proj, vec, pf32, n, g, a, s);
    case HC_DTYPE_F16: return mix_fwd_f16(fused, proj, vec, pf32, n, g, a, s);
    case HC_DTYPE_BF16: return mix_fwd_bf16(fused, proj, vec, pf32, n, g, a, s);
  }
  return HC_ERR_DTYPE;
}

int run_bwd(int sdt, bool fused, bool proj, bool vec, bool pf32, int n, const MixGeometry& g,
            const MixBwdArgs& a, cudaStream_t s) {
  switch (sdt) {
    case HC_DTYPE_F32: return mix_bwd_f32(fused, proj, vec, pf32, n, g, a, s);
    case HC_DTYPE_F16: return mix_bwd_f16(fused, proj, vec, pf32, n, g, a, s);
    case HC_DTYPE_BF16: return mix_bwd_bf16(fused, proj, vec, pf32, n, g, a, s);
  }
  return HC_ERR_DTYPE;
}

bool params_aligned(int pdt, const void* p) { return pdt != HC_DTYPE_F32 || p == nullptr || aligned4(p); }

int run_fwd_tma(int sdt, bool fused, bool proj, bool pf32, int n, const WarpGeometry& g, const MixFwdArgs& a,
                cudaStream_t s) {
  switch (sdt) {
    case HC_DTYPE_F32: return mix_fwd_warp_f32(fused, proj, pf32, n, g, a, s);
    case HC_DTYPE_F16: return mix_fwd_warp_f16(fused, proj, pf32, n, g, a, s);
    case HC_DTYPE_BF16: return mix_fwd_warp_bf16(fused, proj, pf32, n, g, a, s);
  }
  return HC_ERR_DTYPE;
}

int run_bwd_tma(int sdt, bool fused, bool proj, bool pf32, int n, const WarpGeometry& g, const MixBwdArgs& a,
                cudaStream_t s) {
  switch (sdt) {
    case HC_DTYPE_F32: return mix_bwd_warp_f32(fused, proj, pf32, n, g, a, s);
    case HC_DTYPE_F16: return mix_bwd_warp_f16(fused, proj, pf32, n, g, a, s);
    case HC_DTYPE_BF16: return mix_bwd_warp_bf16(fused, proj, pf32, n, g, a, s);
  }
  return HC_ERR_DTYPE;
}

// The pipelined kernels need D % (16 B / element) == 0 (bulk copies move
// multiples of 16 bytes) and 16-byte aligned stream bases.
bool use_tma(bool vec, WarpGeometry& geo, bool bwd, bool fused, bool proj, int n, int64_t T, int64_t D,
             int sdt) {
  return vec && warp_geometry(geo, bwd, fused, proj, n, T, D, dtype_size(sdt), sm_count());
}

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_stream_mix_fwd(const void* Phi, const void* x, const void* Y, const void* v,
                                 void* out, int64_t B, int n, int64_t D, int stream_dtype,
                                 int param_dtype, void* stream) {
  HC_ENTRY("hc_stream_mix_fwd");
  int rc = check_sizes(B, n, D, kBigMaxN);
  if (rc) return rc;
  rc = check_dtypes(stream_dtype, param_dtype);
  if (rc) return rc;
  if (B == 0 || D == 0) return HC_OK;
  if (!Phi || !x || !Y || !out) return HC_ERR_NULL_POINTER;
  if (!params_aligned(param_dtype, Phi) || !params_aligned(param_dtype, v)) return HC_ERR_ALIGNMENT;
  if (n > 8) {  // shared-memory kernels; 32-bit word accesses when every row is word-aligned
    MixFwdArgs a{};
    a.x = x; a.src = Y; a.phi = Phi; a.v = v; a.out = out; a.T = B; a.D = D;
    const bool word = stream_dtype == HC_DTYPE_F32 ||
                      (D % 2 == 0 && aligned4(x) && aligned4(Y) && aligned4(out));
    return run_big_fwd(stream_dtype, v != nullptr, word, param_dtype == HC_DTYPE_F32, n, a,
                       static_cast<cudaStream_t>(stream));
  }
  const int W = vec_width(stream_dtype);
  const bool vec = (D % W == 0) && aligned16(x) && aligned16(Y) && aligned16(out);
  const MixGeometry g = mix_geometry(B, D, vec ? W : 1);
  MixFwdArgs a{};
  a.x = x; a.src = Y; a.phi = Phi; a.v = v; a.out = out;
  a.T = B; a.D = D; a.nchunk = g.nchunk; a.passes = g.passes;
  WarpGeometry geo;
  if (use_tma(vec, geo, false, false, v != nullptr, n, B, D, stream_dtype))
    return run_fwd_tma(stream_dtype, false, v != nullptr, param_dtype == HC_DTYPE_F32, n, geo, a,
                       static_cast<cudaStream_t>(stream));
  return run_fwd(stream_dtype, false, v != nullptr, vec, param_dtype == HC_DTYPE_F32, n, g, a,
                 static_cast<cudaStream_t>(stream));
}

extern "C" int hc_stream_mix_bwd(const void* G, const void* Phi, const void* x, const void* v,
                                 void* grad_x, float* grad_Phi, float* grad_v, int64_t B, int n,
                                 int64_t D, int stream_dtype, int param_dtype, void* stream) {
  HC_ENTRY("hc_stream_mix_bwd");
  int rc = check_sizes(B, n, D, kBigMaxN);
  if (rc) return rc;
  rc = check_dtypes(stream_dtype, param_dtype);
  if (rc) return rc;
  if (B == 0) return HC_OK;
  if (!Phi) return HC_ERR_NULL_POINTER;
  if (D > 0 && (!G || !x)) return HC_ERR_NULL_POINTER;
  if (!params_aligned(param_dtype, Phi) || !params_aligned(param_dtype, v)) return HC_ERR_ALIGNMENT;
  if ((grad_Phi && !aligned4(grad_Phi)) || (grad_v && !aligned4(grad_v))) return HC_ERR_ALIGNMENT;
  if (v == nullptr) grad_v = nullptr;
  if (n > 8) {  // D == 0 still writes the (all-zero) parameter gradients
    MixBwdArgs a{};
    a.g = G; a.x = x; a.phi = Phi; a.v = v;
    a.grad_x = D > 0 ? grad_x : nullptr; a.grad_phi = grad_Phi; a.grad_v = grad_v;
    a.T = B; a.D = D;
    return run_big_bwd(stream_dtype, v != nullptr, param_dtype == HC_DTYPE_F32, n, a,
                       static_cast<cudaStream_t>(stream));
  }
  const int W = vec_width(stream_dtype);
  const bool vec = (D % W == 0) && aligned16(G) && aligned16(x) && (grad_x == nullptr || aligned16(grad_x));
  const MixGeometry g = mix_geometry(B, D, vec ? W : 1);
  MixBwdArgs a{};
  a.g = G; a.x = x; a.phi = Phi; a.v = v;
  a.grad_x = D > 0 ? grad_x : nullptr; a.grad_phi = grad_Phi; a.grad_v = grad_v;
  a.T = B; a.D = D; a.nchunk = g.nchunk; a.passes = g.passes;
  WarpGeometry geo;
  if (use_tma(vec, geo, true, false, v != nullptr, n, B, D, stream_dtype))
    return run_bwd_tma(stream_dtype, false, v != nullptr, param_dtype == HC_DTYPE_F32, n, geo, a,
                       static_cast<cudaStream_t>(stream));
  // D == 0 still writes the (all-zero) parameter gradients.
  return run_bwd(stream_dtype, false, v != nullptr, vec, param_dtype == HC_DTYPE_F32, n, g, a,
                 static_cast<cudaStream_t>(stream));
}

extern "C" int hc_fused_fwd(const void* x, const void* f, const float* H, const float* alpha,
                            const float* beta, void* u, void* x_out, int64_t T, int n, int64_t D,
                            int stream_dtype, void* stream) {
  HC_ENTRY("hc_fused_fwd");
  int rc = check_sizes(T, n, D);
  if (rc) return rc;
  if (dtype_size(stream_dtype) == 0) return HC_ERR_DTYPE;
  if (T == 0 || D == 0) return HC_OK;
  if (!x || !f || !H || !alpha || !beta || !u || !x_out) return HC_ERR_NULL_POINTER;
  if (!aligned4(H) || !aligned4(alpha) || !aligned4(beta)) return HC_ERR_ALIGNMENT;
  const int W = vec_width(stream_dtype);
  const bool vec = (D % W == 0) && aligned16(x) && aligned16(f) && aligned16(u) && aligned16(x_out);
  const MixGeometry g = mix_geometry(T, D, vec ? W : 1);
  MixFwdArgs a{};
  a.x = x; a.src = f; a.phi = H; a.alpha = alpha; a.beta = beta; a.out = x_out; a.u = u;
  a.T = T; a.D = D; a.nchunk = g.nchunk; a.passes = g.passes;
  WarpGeometry geo;
  if (use_tma(vec, geo, false, true, false, n, T, D, stream_dtype))
    return run_fwd_tma(stream_dtype, true, false, true, n, geo, a, static_cast<cudaStream_t>(stream));
  return run_fwd(stream_dtype, true, false, vec, true, n, g, a, static_cast<cudaStream_t>(stream));
}

extern "C" int hc_fused_bwd(const void* g_u, const void* g_x, const void* x, const void* f,
                            const float* H, const float* alpha, const float* beta, void* grad_x,
                            void* grad_f, float* grad_H, float* grad_alpha, float* grad_beta,
                            int64_t T, int n, int64_t D, int stream_dtype, void* stream) {
  HC_ENTRY("hc_fused_bwd");
  int rc = check_sizes(T, n, D);
  if (rc) return rc;
  if (dtype_size(stream_dtype) == 0) return HC_ERR_DTYPE;
  if (T == 0) return HC_OK;
  if (!H || !alpha || !beta) return HC_ERR_NULL_POINTER;
  if (D > 0 && (!g_u || !g_x || !x || !f)) return HC_ERR_NULL_POINTER;
  if (!aligned4(H) || !aligned4(alpha) || !aligned4(beta)) return HC_ERR_ALIGNMENT;
  if ((grad_H && !aligned4(grad_H)) || (grad_alpha && !aligned4(grad_alpha)) ||
      (grad_beta && !aligned4(grad_beta)))
    return HC_ERR_ALIGNMENT;
  const int W = vec_width(stream_dtype);
  const bool vec = (D % W == 0) && aligned16(g_u) && aligned16(g_x) && aligned16(x) && aligned16(f) &&
                   (grad_x == nullptr || aligned16(grad_x)) && (grad_f == nullptr || aligned16(grad_f));
  const MixGeometry g = mix_geometry(T, D, vec ? W : 1);
  MixBwdArgs a{};
  a.g = g_x; a.gu = g_u; a.x = x; a.f = f; a.phi = H; a.alpha = alpha; a.beta = beta;
  a.grad_x = D > 0 ? grad_x : nullptr; a.grad_f = D > 0 ? grad_f : nullptr;
  a.grad_phi = grad_H; a.grad_alpha = grad_alpha; a.grad_beta = grad_beta;
  a.T = T; a.D = D; a.nchunk = g.nchunk; a.passes = g.passes;
  WarpGeometry geo;
  if (use_tma(vec, geo, true, true, false, n, T, D, stream_dtype))
    return run_bwd_tma(stream_dtype, true, false, true, n, geo, a, static_cast<cudaStream_t>(stream));
  return run_bwd(stream_dtype, true, false, vec, true, n, g, a, static_cast<cudaStream_t>(stream));
}

extern "C" int hc_wait_timeouts(unsigned int* count, int reset) {
  if (!count) return HC_ERR_NULL_POINTER;
  if (cudaDeviceSynchronize() != cudaSuccess) return HC_ERR_LAUNCH;
  const bool r = reset != 0;
  *count = mix_warp_take_timeouts_f32(r) + mix_warp_take_timeouts_f16(r) + mix_warp_take_timeouts_bf16(r) +
           rw_fwd_take_timeouts_f32(r) + rw_fwd_take_timeouts_f16(r) + rw_fwd_take_timeouts_bf16(r) +
           rw_bwd_take_timeouts_f32(r) + rw_bwd_take_timeouts_f16(r) + rw_bwd_take_timeouts_bf16(r) +
           expm_take_timeouts(r);
  if (r) clear_timeout_word();
  return HC_OK;
}
