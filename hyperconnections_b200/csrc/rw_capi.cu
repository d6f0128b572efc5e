// rw_capi.cu — C entry points of the width-read and mix + depth-write kernels
// for a general backbone width m (see hcops.h).
//
// Host-side checks come first (sizes, dtype, NULL pointers, alignment). The
// ring kernels run when 1 <= m <= min(n, 4), D is a multiple of 16 bytes of
// elements and every stream base is 16-byte aligned; any other shape runs
// the element-wise kernels of the same arithmetic.
#include "rw_warp.cuh"
#include "bign_ring.cuh"  // big_ring_geometry (hc_debug_ring_geometry)

namespace hc {
namespace {

constexpr int64_t kMaxD = int64_t(1) << 24;
constexpr int64_t kMaxTokens = (int64_t(1) << 31) - 1;

int check_rw(int64_t T, int n, int m, int64_t D, int sdt) {
  if (T < 0 || T > kMaxTokens || D < 0 || D > kMaxD) return HC_ERR_BAD_SIZE;
  if (n < 1 || n > 8 || m < 1 || m > 4) return HC_ERR_UNSUPPORTED_N;
  if (dtype_size(sdt) == 0) return HC_ERR_DTYPE;
  return HC_OK;
}

bool f32_aligned(const float* p) { return p == nullptr || aligned4(p); }

bool stream_ok(const void* p) { return p == nullptr || aligned16(p); }

int dispatch(bool bwd, int sdt, bool ring, bool mixw, bool proj, int n, int m, const WarpGeometry& g,
             const RwArgs& a, cudaStream_t s) {
  switch (sdt) {
    case HC_DTYPE_F32: return bwd ? rw_bwd_f32(ring, mixw, proj, n, m, g, a, s) : rw_fwd_f32(ring, mixw, proj, n, m, g, a, s);
    case HC_DTYPE_F16: return bwd ? rw_bwd_f16(ring, mixw, proj, n, m, g, a, s) : rw_fwd_f16(ring, mixw, proj, n, m, g, a, s);
    case HC_DTYPE_BF16: return bwd ? rw_bwd_bf16(ring, mixw, proj, n, m, g, a, s) : rw_fwd_bf16(ring, mixw, proj, n, m, g, a, s);
  }
  return HC_ERR_DTYPE;
}

// Ring geometry when the shape and the pointers allow it.
bool ring_ok(WarpGeometry& geo, bool bwd, bool mixw, bool proj, int n, int m, int64_t T, int64_t D, int sdt,
             bool streams_aligned) {
  const int es = dtype_size(sdt);
  if (!streams_aligned || !rw_ring_supported(n, m) || D % (16 / es) != 0) return false;
  const int cap = rw_cap(bwd, n, m, mixw, proj);
  const int rows = rw_rows(bwd, n, m, mixw);
  // the read rings group small tokens into items of up to 20 KB: measured on
  // B200 (16,384 tokens, bf16) against the fused step's 15 / 16 KB, read
  // forward +49% at n = 2, D = 2048, +23% at n = 4, m = 1, D = 768, +13% at
  // m = 2 (-3% at n = 4, m = 4, D = 512); read backward +28% at n = 4, m = 2,
  // D = 768, within 1% elsewhere
  const int64_t item = mixw ? 0 : 20 * 1024;
  if (!ring_geometry(geo, rows, cap, T, D, es, sm_count(), bwd, item)) return false;
  if (bwd && geo.ns > 1 && rw_gram_mma(n, mixw, es)) {
    // the Gram on the tensor cores (rw_gram_finish), on swizzled or padded stages
    const WarpGeometry plain = geo;
    rw_mma_geometry(geo, plain, n, m, T, D, es, true);
  }
  if (bwd && (cap > 8 || geo.gram_mma)) prefer_bwd_consumers(geo, 4);
  if (mixw) {
    prefer_producers(geo);
  } else if (mix_tuning().producers > 0) {
    geo.producers = std::min(mix_tuning().producers, geo.stages);
  }
  if (bwd && mixw && !proj && (n == 2 || n == 4) && geo.ns == 1 && geo.tpi == 1 && !geo.gram_mma && HC_BWD_SIDE) {
    // side rows of f (rw_side_fetch): stages of the 2n rows of g and x, then
    // two slots of f rows per consumer; consumers trimmed (at most two) where
    // the slots would leave fewer than consumers + 2 stages. Measured on B200
    // (16,384 tokens, bf16, mix-write backward) against the plain ring:
    // n = 4, m = 1, D = 768 73.9 -> 68.5 us; n = 4, m = 2, D = 768 76.6 ->
    // 71.5 us; n = 2, m = 1, D = 2048 93.8 -> 91.7 us; n = 4, m = 4, D = 512
    // level; n = 4, m = 1, D = 1024 80.0 -> 83.3 us (a loss kept with the
    // rule); with the projection 78.7 -> 80.5 us, so not taken there.
    WarpGeometry sg = geo;
    const int slot2 = 2 * m * static_cast<int>(D) * es;  // a consumer's two slots
    sg.stage_bytes = 2 * n * sg.pitch * es;
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
  return true;
}

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_read_fwd(const float* R, const void* x, void* u, int64_t T, int n, int m, int64_t D,
                           int stream_dtype, void* stream) {
  HC_ENTRY("hc_read_fwd");
  int rc = check_rw(T, n, m, D, stream_dtype);
  if (rc) return rc;
  if (T == 0 || D == 0) return HC_OK;
  if (!R || !x || !u) return HC_ERR_NULL_POINTER;
  if (!f32_aligned(R)) return HC_ERR_ALIGNMENT;
  RwArgs a{};
  a.x = x; a.R = R; a.out = u; a.T = T; a.D = D;
  WarpGeometry geo{};
  const bool ring = ring_ok(geo, false, false, false, n, m, T, D, stream_dtype, aligned16(x) && aligned16(u));
  return dispatch(false, stream_dtype, ring, false, false, n, m, geo, a, static_cast<cudaStream_t>(stream));
}

extern "C" int hc_read_bwd(const void* g_u, const float* R, const void* x, void* grad_x, float* grad_R, int64_t T,
                           int n, int m, int64_t D, int stream_dtype, void* stream) {
  HC_ENTRY("hc_read_bwd");
  int rc = check_rw(T, n, m, D, stream_dtype);
  if (rc) return rc;
  if (T == 0) return HC_OK;
  if (!R) return HC_ERR_NULL_POINTER;
  if (D > 0 && (!g_u || !x)) return HC_ERR_NULL_POINTER;
  if (!f32_aligned(R) || !f32_aligned(grad_R)) return HC_ERR_ALIGNMENT;
  RwArgs a{};
  a.g = g_u; a.x = x; a.R = R; a.grad_x = D > 0 ? grad_x : nullptr; a.grad_R = grad_R; a.T = T; a.D = D;
  WarpGeometry geo{};
  const bool ring = ring_ok(geo, true, false, false, n, m, T, D, stream_dtype,
                            aligned16(g_u) && aligned16(x) && stream_ok(grad_x));
  // D == 0 still writes the (all-zero) grad_R through the element-wise kernel.
  return dispatch(true, stream_dtype, ring, false, false, n, m, geo, a, static_cast<cudaStream_t>(stream));
}

extern "C" int hc_mix_write_fwd(const float* H, const void* x, const float* W, const void* f, const float* v,
                                void* out, int64_t T, int n, int m, int64_t D, int stream_dtype, void* stream) {
  HC_ENTRY("hc_mix_write_fwd");
  int rc = check_rw(T, n, m, D, stream_dtype);
  if (rc) return rc;
  if (T == 0 || D == 0) return HC_OK;
  if (!H || !x || !W || !f || !out) return HC_ERR_NULL_POINTER;
  if (!f32_aligned(H) || !f32_aligned(W) || !f32_aligned(v)) return HC_ERR_ALIGNMENT;
  RwArgs a{};
  a.x = x; a.f = f; a.H = H; a.W = W; a.v = v; a.out = out; a.T = T; a.D = D;
  const bool proj = v != nullptr;
  WarpGeometry geo{};
  const bool ring = ring_ok(geo, false, true, proj, n, m, T, D, stream_dtype,
                            aligned16(x) && aligned16(f) && aligned16(out));
  return dispatch(false, stream_dtype, ring, true, proj, n, m, geo, a, static_cast<cudaStream_t>(stream));
}

extern "C" int hc_mix_write_bwd(const void* g, const float* H, const void* x, const float* W, const void* f,
                                const float* v, void* grad_x, void* grad_f, float* grad_H, float* grad_W,
                                float* grad_v, int64_t T, int n, int m, int64_t D, int stream_dtype, void* stream) {
  HC_ENTRY("hc_mix_write_bwd");
  int rc = check_rw(T, n, m, D, stream_dtype);
  if (rc) return rc;
  if (T == 0) return HC_OK;
  if (!H || !W) return HC_ERR_NULL_POINTER;
  if (D > 0 && (!g || !x || !f)) return HC_ERR_NULL_POINTER;
  if (!f32_aligned(H) || !f32_aligned(W) || !f32_aligned(v) || !f32_aligned(grad_H) || !f32_aligned(grad_W) ||
      !f32_aligned(grad_v))
    return HC_ERR_ALIGNMENT;
  RwArgs a{};
  a.g = g; a.x = x; a.f = f; a.H = H; a.W = W; a.v = v;
  a.grad_x = D > 0 ? grad_x : nullptr; a.grad_f = D > 0 ? grad_f : nullptr;
  a.grad_H = grad_H; a.grad_W = grad_W; a.grad_v = v ? grad_v : nullptr; a.T = T; a.D = D;
  const bool proj = v != nullptr;
  WarpGeometry geo{};
  const bool ring = ring_ok(geo, true, true, proj, n, m, T, D, stream_dtype,
                            aligned16(g) && aligned16(x) && aligned16(f) && stream_ok(grad_x) && stream_ok(grad_f));
  return dispatch(true, stream_dtype, ring, true, proj, n, m, geo, a, static_cast<cudaStream_t>(stream));
}

extern "C" int hc_debug_ring_geometry(int op, int bwd, int n, int m, int proj, int64_t T, int64_t D,
                                      int stream_dtype, int* out, int out_len) {
  if (!out) return HC_ERR_NULL_POINTER;
  if (out_len < 1) return HC_ERR_BAD_SIZE;
  if (stream_dtype != HC_DTYPE_F32 && stream_dtype != HC_DTYPE_F16 && stream_dtype != HC_DTYPE_BF16)
    return HC_ERR_DTYPE;
  if (T <= 0 || D <= 0) return HC_ERR_BAD_SIZE;
  const int es = dtype_size(stream_dtype);
  WarpGeometry geo{};
  bool ring = false;
  switch (op) {
    case 0:  // the fused step (m = 1, no projection)
    case 1:  // stream_mix_add
      if (op == 1 && n > 8 && n <= kBigMaxN) {  // 9 <= n <= 32: the tensor-core ring (half precision)
        ring = es == 2 && HC_GRAM_MMA && big_ring_geometry(geo, n, T, D);
        break;
      }
      if (n < 1 || n > 8) return HC_ERR_UNSUPPORTED_N;
      ring = D % (16 / es) == 0 &&
             warp_geometry(geo, bwd != 0, op == 0, op == 1 && proj != 0, n, T, D, es, sm_count());
      break;
    case 2:  // read
    case 3:  // mix-write
      if (int rc = check_rw(T, n, m, D, stream_dtype)) return rc;
      ring = ring_ok(geo, bwd != 0, op == 3, op == 3 && proj != 0, n, m, T, D, stream_dtype, true);
      break;
    default:
      return HC_ERR_BAD_SIZE;
  }
  const int v[12] = {ring ? 1 : 0, geo.stages, geo.consumers, geo.producers, geo.tpi, geo.sl,
                     geo.ns, geo.stage_bytes, geo.smem_bytes, geo.side, geo.gram_mma, geo.grid};
  for (int i = 0; i < out_len && i < 12; ++i) out[i] = ring ? v[i] : 0;
  return HC_OK;
}
