// bign_ring.cuh — stream_mix_add for 9 <= n <= 32 streams with
// half-precision streams, backward and forward, on the shared-memory ring of
// mix_warp.cuh and the tensor cores.
//
// Same arithmetic as big_bwd_kernel (bign.cuh; reference
// ops/stream_mix_small_nb.py:341-391 and stream_mix_big_nb.py for N >= 16):
//   grad_x_j   = sum_i Phi_ij G_i [+ v_j (c^T G)] = (Phi' ^T G)_j,  Phi' = Phi [+ c v^T]
//   grad_Phi_ij = M_ij [- v_j rho_i],  M = G x^T summed over D (the Gram)
//   grad_v_j   = rho_j - sum_i Phi_ij rho_i + bp_j,
//   rho_i = sum_j v_j M_ij,  bp_j = sum_i c_i M_ij,  c = v - Phi v.
//
// A persistent CTA per SM owns a contiguous range of tokens; warp 0 fills the
// ring with slices of one token (its n rows of G and of x, one TMA tensor copy
// each, on the swizzled stages of the tensor-core Gram: a row holds an odd
// number of 128-byte lines, so 8 rows of one 16-byte column fall in 8
// different bank groups). A token stays on one consumer warp, which per
// 16-element step of a slice
//   * loads the G rows with ldmatrix twice: as the A operand of the Gram
//     (rows i, k = elements) and, transposed, as the B operand of grad_x
//     (k = rows i, n = elements), and the x rows as the Gram's B operand;
//   * accumulates the Gram M (n x n, fp32, in registers over the token's
//     slices) with mma.sync.m16n8k16: the product of two half-precision
//     values is exact in fp32;
//   * forms grad_x = Phi'^T G for the step's 16 elements with Phi'^T as the A
//     operand split in two half-precision parts, hi = round(Phi'^T) and
//     lo = round(Phi'^T - hi), so that the operand carries ~16 significant
//     bits (the result is rounded to the stream type once, from fp32), and
//     stores it straight from the accumulators (4-byte words, every byte of
//     grad_x written once).
// At the token's last slice the finish folds M into grad_Phi and grad_v
// (quad and column shuffles of the accumulator layout, two small per-warp
// arrays in shared memory).
#pragma once

#include "bign.cuh"

namespace hc {

constexpr int kBigRingWarps = 8;  // producer + 7 consumers (255 registers a thread)

template <int NMAX>
struct BigMma {
  static constexpr int MT = NMAX / 16;  // 16-row tiles over n
  static constexpr int NT = NMAX / 8;   // 8-column tiles of the Gram
};

template <typename T>
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Two fp32 values as one 32-bit word of the stream type (low half first).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const float f[2] = {lo, hi};
  return Word<T>::put(f);
}

// A value split into two half-precision parts hi + lo (hi = round(a),
// lo = round(a - hi)).
template <typename T>
__device__ __forceinline__ void split2(float a, float& hi, float& lo) {
  hi = Elem<T>::to_f(Elem<T>::from_f(a));
  lo = a - hi;
}

// Per-token operands of one consumer warp: the A fragments of Phi'^T
// (hi and lo parts) for every (row tile, k tile).
template <int NMAX>
struct BigTokA {
  static constexpr int MT = BigMma<NMAX>::MT;
  uint32_t hi[MT][MT][4], lo[MT][MT][4];
};

// Loads token t's Phi (and v, c = v - Phi v) and builds the A fragments of
// Phi'^T: register r of tile (mt, ks) holds rows j = 16 mt + lane / 4 (+8 for
// r odd) and columns i = 16 ks + 2 (lane % 4) (+8 for r >= 2), two columns a
// word. vs / cs: the warp's v and c (NMAX floats each, zero past n).
// (TRANS = false: the A fragments of Phi' itself, rows i and columns j, for
// the forward.)
template <typename T, typename P, int NMAX, bool PROJ, bool TRANS = true>
__device__ __forceinline__ void big_tok_load(const void* phi, const void* v, int64_t t, int n, BigTokA<NMAX>& A,
                                             float* vs, float* cs, int lane) {
  constexpr int MT = BigMma<NMAX>::MT;
  const P* ph = static_cast<const P*>(phi) + t * n * n;
  if constexpr (PROJ) {
    const P* vp = static_cast<const P*>(v) + t * n;
    if (lane < NMAX) vs[lane] = lane < n ? Elem<P>::to_f(vp[lane]) : 0.f;
    __syncwarp();
    if (lane < NMAX) {
      float pv = 0.f;
      if (lane < n)
        for (int j = 0; j < n; ++j) pv = fmaf(Elem<P>::to_f(ph[lane * n + j]), vs[j], pv);
      cs[lane] = lane < n ? vs[lane] - pv : 0.f;
    }
    __syncwarp();
  }
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int ks = 0; ks < MT; ++ks) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = 16 * mt + g + ((r & 1) ? 8 : 0);
        float h[2], l[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = 16 * ks + 2 * q + ((r & 2) ? 8 : 0) + e;
          const int i = TRANS ? col : row, j = TRANS ? row : col;  // Phi'_ij = Phi_ij + c_i v_j
          float val = 0.f;
          if (i < n && j < n) {
            val = Elem<P>::to_f(ph[i * n + j]);
            if constexpr (PROJ) val = fmaf(cs[i], vs[j], val);
          }
          split2<T>(val, h[e], l[e]);
        }
        A.hi[mt][ks][r] = pack2<T>(h[0], h[1]);
        A.lo[mt][ks][r] = pack2<T>(l[0], l[1]);
      }
    }
  }
}

// One slice of a token: the Gram into gram, grad_x of the slice's elements to
// global memory. gs / xs: the stage's swizzled regions of G and x (n rows, nc
// lines a row); len: the slice's elements (a multiple of 64).
template <typename T, int NMAX>
__device__ __forceinline__ void big_slice(float (&gram)[BigMma<NMAX>::MT][BigMma<NMAX>::NT][4],
                                          const BigTokA<NMAX>& A, const uint8_t* gs, const uint8_t* xs,
                                          const uint8_t* zrow, int nc, int n, int len, T* gxt, int64_t D,
                                          int lane) {
  constexpr int MT = BigMma<NMAX>::MT, NT = BigMma<NMAX>::NT;
  constexpr int es = sizeof(T);
  const int q = lane >> 3;
  const int g = lane >> 2, qd = lane & 3;
  const uint32_t z = smem_u32(zrow);
  // row of this lane's ldmatrix address in each 16-row tile: A / trans-B
  // (rows (q & 1) * 8 + lane % 8, elements (q >> 1) * 8), and B of the Gram
  // (rows (q >> 1) * 8 + lane % 8, elements (q & 1) * 8)
  const int ar = (q & 1) * 8 + (lane & 7), akof = (q >> 1) * 8;
  const int br = (q >> 1) * 8 + (lane & 7), bkof = (q & 1) * 8;
  for (int k0 = 0; k0 < len; k0 += 16) {
    uint32_t ga[MT][4], gt[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int i = 16 * mt + ar;
      const uint32_t addr = i < n ? smem_u32(swz_at(gs, nc, i, (k0 + akof) * es)) : z;
      ldsm_x4(ga[mt], addr);
      ldsm_x4_trans<T>(gt[mt], addr);
    }
    // the Gram: M[i][j] += G_i . x_j over these 16 elements
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      const int j = 16 * np + br;
      uint32_t xb[4];
      ldsm_x4(xb, j < n ? smem_u32(swz_at(xs, nc, j, (k0 + bkof) * es)) : z);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        MmaKind<T>::mma(gram[mt][2 * np], ga[mt], xb[0], xb[1]);
        MmaKind<T>::mma(gram[mt][2 * np + 1], ga[mt], xb[2], xb[3]);
      }
    }
    // grad_x rows j, elements k0 .. k0 + 15 (two 8-column tiles)
    if (gxt) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        float c[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) c[h][0] = c[h][1] = c[h][2] = c[h][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < MT; ++ks) {
          // trans-B of k tile ks: gt[ks][0..1] -> elements k0..k0+7, [2..3] -> k0+8..k0+15
          MmaKind<T>::mma(c[0], A.hi[mt][ks], gt[ks][0], gt[ks][1]);
          MmaKind<T>::mma(c[0], A.lo[mt][ks], gt[ks][0], gt[ks][1]);
          MmaKind<T>::mma(c[1], A.hi[mt][ks], gt[ks][2], gt[ks][3]);
          MmaKind<T>::mma(c[1], A.lo[mt][ks], gt[ks][2], gt[ks][3]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int64_t col = k0 + 8 * h + 2 * qd;
          const int j0 = 16 * mt + g;
          if (j0 < n) *reinterpret_cast<uint32_t*>(gxt + j0 * D + col) = pack2<T>(c[h][0], c[h][1]);
          if (j0 + 8 < n) *reinterpret_cast<uint32_t*>(gxt + (j0 + 8) * D + col) = pack2<T>(c[h][2], c[h][3]);
        }
      }
    }
  }
}

// The token's grad_Phi and grad_v from its Gram (accumulator layout: tile
// (mt, nt) register e holds row i = 16 mt + lane / 4 (+8 for e >= 2) and
// column j = 8 nt + 2 (lane % 4) + (e & 1)). rs / bs: the warp's rho and bp
// (NMAX floats each).
template <typename P, int NMAX, bool PROJ>
__device__ __forceinline__ void big_finish(const MixBwdArgs& a, const float (&gram)[BigMma<NMAX>::MT][BigMma<NMAX>::NT][4],
                                           int64_t t, int n, const float* vs, const float* cs, float* rs, float* bs,
                                           int lane) {
  constexpr int MT = BigMma<NMAX>::MT, NT = BigMma<NMAX>::NT;
  const int g = lane >> 2, qd = lane & 3;
  float rho[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) rho[mt][0] = rho[mt][1] = 0.f;
  if constexpr (PROJ) {
    float bp[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) bp[nt][0] = bp[nt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 16 * mt + g + (e >= 2 ? 8 : 0), j = 8 * nt + 2 * qd + (e & 1);
          rho[mt][e >> 1] = fmaf(vs[j], gram[mt][nt][e], rho[mt][e >> 1]);
          bp[nt][e & 1] = fmaf(cs[i], gram[mt][nt][e], bp[nt][e & 1]);
        }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        rho[mt][h] += __shfl_xor_sync(kFull, rho[mt][h], 1);
        rho[mt][h] += __shfl_xor_sync(kFull, rho[mt][h], 2);
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        bp[nt][e] += __shfl_xor_sync(kFull, bp[nt][e], 4);
        bp[nt][e] += __shfl_xor_sync(kFull, bp[nt][e], 8);
        bp[nt][e] += __shfl_xor_sync(kFull, bp[nt][e], 16);
      }
    if (qd == 0) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        rs[16 * mt + g] = rho[mt][0];
        rs[16 * mt + g + 8] = rho[mt][1];
      }
    }
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        bs[8 * nt + 2 * qd] = bp[nt][0];
        bs[8 * nt + 2 * qd + 1] = bp[nt][1];
      }
    }
  }
  if (a.grad_phi) {
    float* gp = a.grad_phi + t * n * n;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 16 * mt + g + (e >= 2 ? 8 : 0), j = 8 * nt + 2 * qd + (e & 1);
          float val = gram[mt][nt][e];
          if constexpr (PROJ) val = fmaf(-vs[j], rho[mt][e >> 1], val);
          if (i < n && j < n) gp[i * n + j] = val;
        }
  }
  if constexpr (PROJ) {
    __syncwarp();
    if (a.grad_v && lane < n) {
      const P* ph = static_cast<const P*>(a.phi) + t * n * n;
      float ht = 0.f;
      for (int i = 0; i < n; ++i) ht = fmaf(Elem<P>::to_f(ph[i * n + lane]), rs[i], ht);
      a.grad_v[t * n + lane] = (rs[lane] - ht) + bs[lane];
    }
  }
  __syncwarp();
}

template <typename T, typename P, int NMAX, bool PROJ>
__global__ void __launch_bounds__(kBigRingWarps * 32, 1)
big_bwd_ring_kernel(const MixBwdArgs a, const WarpGeometry geo, const __grid_constant__ RingMaps maps, int n) {
  static_assert(sizeof(T) == 2, "half-precision streams");
  constexpr int MT = BigMma<NMAX>::MT, NT = BigMma<NMAX>::NT;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // swizzled stages start on a 1024-byte boundary (kSwzAlign bytes of slack)
  uint8_t* const smem = smem_raw + ((kSwzAlign - (smem_u32(smem_raw) & (kSwzAlign - 1))) & (kSwzAlign - 1));
  __shared__ RingState st;
  __shared__ float warp_vec[kBigRingWarps - 1][4][NMAX];  // per consumer: v, c, rho, bp
  pdl_launch_dependents();
  ring_init(st, geo.stages);
  pdl_wait_prior_grid();

  const int64_t T_ = a.T, D = a.D;
  const UnitMap um = unit_map(T_, 1);
  const int ntok = um.nunits;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = geo.stages, C = geo.consumers, ns = geo.ns;
  const int nc = geo.sl / kTmaChunk;
  const int rn = swz_region_bytes(n, geo.sl, 2);

  if (warp == 0) {
    if (lane < geo.producers) {
      const void* base[2] = {a.g, a.x};
      const int rows[2] = {n, n};
      ring_produce<T, 2>(st, geo, smem, D, um, base, rows, lane, &maps);
    }
  } else if (warp - 1 < C) {
    const int c = warp - 1;
    float* vs = warp_vec[c][0];
    float* cs = warp_vec[c][1];
    float* rs = warp_vec[c][2];
    float* bs = warp_vec[c][3];
    BigTokA<NMAX> A;
    float gram[MT][NT][4];
    RingCursor cur{c, 0u, c};
    for (int g0 = 0; g0 < ntok; g0 += C) {
      const int Wg = min(C, ntok - g0);
      if (c >= Wg) break;
      const int64_t t = um.tok(g0 + c);
      big_tok_load<T, P, NMAX, PROJ>(a.phi, a.v, t, n, A, vs, cs, lane);  // overlaps the wait for the data
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) gram[mt][nt][0] = gram[mt][nt][1] = gram[mt][nt][2] = gram[mt][nt][3] = 0.f;
      T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * n * D : nullptr;
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
        big_slice<T, NMAX>(gram, A, sb, sb + rn, reinterpret_cast<const uint8_t*>(st.zrow), nc, n, len,
                           gxt ? gxt + d0 : nullptr, D, lane);
        if (p == ns - 1) big_finish<P, NMAX, PROJ>(a, gram, t, n, vs, cs, rs, bs, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&st.empty[cur.s]);
        cur.advance(p + 1 < ns ? Wg : C, S);
      }
      if (!ok) break;
    }
  }
  ring_drain(st, S);
}

// ------------------------------------------------------------------ forward
// out_i = sum_j Phi'_ij x_j + Y_i (Phi' = Phi [+ c v^T]; reference
// ops/stream_mix_small_nb.py:75-132): the ring holds a slice of the token's x
// and Y rows (swizzled stages as above); per 16-element step the consumer
// loads the x rows transposed as the B operand, multiplies by Phi' (A operand,
// hi / lo split, registers), adds Y from the stage to the fp32 accumulators
// and stores out straight from them.
template <typename T, int NMAX>
__device__ __forceinline__ void big_fwd_slice(const BigTokA<NMAX>& A, const uint8_t* xs, const uint8_t* ys,
                                              const uint8_t* zrow, int nc, int n, int len, T* ot, int64_t D,
                                              int lane) {
  constexpr int MT = BigMma<NMAX>::MT;
  constexpr int es = sizeof(T);
  const int q = lane >> 3;
  const int g = lane >> 2, qd = lane & 3;
  const uint32_t z = smem_u32(zrow);
  const int ar = (q & 1) * 8 + (lane & 7), akof = (q >> 1) * 8;
  for (int k0 = 0; k0 < len; k0 += 16) {
    uint32_t xt[MT][4];
#pragma unroll
    for (int ks = 0; ks < MT; ++ks) {
      const int j = 16 * ks + ar;
      ldsm_x4_trans<T>(xt[ks], j < n ? smem_u32(swz_at(xs, nc, j, (k0 + akof) * es)) : z);
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float c[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) c[h][0] = c[h][1] = c[h][2] = c[h][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < MT; ++ks) {
        MmaKind<T>::mma(c[0], A.hi[mt][ks], xt[ks][0], xt[ks][1]);
        MmaKind<T>::mma(c[0], A.lo[mt][ks], xt[ks][0], xt[ks][1]);
        MmaKind<T>::mma(c[1], A.hi[mt][ks], xt[ks][2], xt[ks][3]);
        MmaKind<T>::mma(c[1], A.lo[mt][ks], xt[ks][2], xt[ks][3]);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = k0 + 8 * h + 2 * qd;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int i = 16 * mt + g + 8 * hr;
          if (i < n) {
            float y[2];
            Word<T>::get(*reinterpret_cast<const uint32_t*>(swz_at(ys, nc, i, col * es)), y);
            *reinterpret_cast<uint32_t*>(ot + i * D + col) =
                pack2<T>(c[h][2 * hr] + y[0], c[h][2 * hr + 1] + y[1]);
          }
        }
      }
    }
  }
}

template <typename T, typename P, int NMAX, bool PROJ>
__global__ void __launch_bounds__(kBigRingWarps * 32, 1)
big_fwd_ring_kernel(const MixFwdArgs a, const WarpGeometry geo, const __grid_constant__ RingMaps maps, int n) {
  static_assert(sizeof(T) == 2, "half-precision streams");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* const smem = smem_raw + ((kSwzAlign - (smem_u32(smem_raw) & (kSwzAlign - 1))) & (kSwzAlign - 1));
  __shared__ RingState st;
  __shared__ float warp_vec[kBigRingWarps - 1][2][NMAX];  // per consumer: v, c
  pdl_launch_dependents();
  ring_init(st, geo.stages);
  pdl_wait_prior_grid();

  const int64_t T_ = a.T, D = a.D;
  const UnitMap um = unit_map(T_, 1);
  const int ntok = um.nunits;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = geo.stages, C = geo.consumers, ns = geo.ns;
  const int nc = geo.sl / kTmaChunk;
  const int rn = swz_region_bytes(n, geo.sl, 2);

  if (warp == 0) {
    if (lane < geo.producers) {
      const void* base[2] = {a.x, a.src};
      const int rows[2] = {n, n};
      ring_produce<T, 2>(st, geo, smem, D, um, base, rows, lane, &maps);
    }
  } else if (warp - 1 < C) {
    const int c = warp - 1;
    BigTokA<NMAX> A;
    RingCursor cur{c, 0u, c};
    for (int g0 = 0; g0 < ntok; g0 += C) {
      const int Wg = min(C, ntok - g0);
      if (c >= Wg) break;
      const int64_t t = um.tok(g0 + c);
      big_tok_load<T, P, NMAX, PROJ, false>(a.phi, a.v, t, n, A, warp_vec[c][0], warp_vec[c][1], lane);
      T* ot = static_cast<T*>(a.out) + t * n * D;
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
        big_fwd_slice<T, NMAX>(A, sb, sb + rn, reinterpret_cast<const uint8_t*>(st.zrow), nc, n, len, ot + d0, D,
                               lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&st.empty[cur.s]);
        cur.advance(p + 1 < ns ? Wg : C, S);
      }
      if (!ok) break;
    }
  }
  ring_drain(st, S);
}

// Ring geometry of the kernels above for two tensors of n rows a token: slices
// of an odd number of 64-element chunks (at most the chunks that let 9 stages
// fit the ring), split as evenly as that allows; false when the shape does
// not fit (the caller then runs big_bwd_kernel).
inline bool big_ring_geometry(WarpGeometry& geo, int n, int64_t T, int64_t D) {
  if (n < 9 || n > kBigMaxN || T <= 0 || D <= 0 || D % kTmaChunk != 0 || T * n >= (int64_t(1) << 31)) return false;
  // stages of at most kGramBudget / 9 bytes: 9 stages, 7 consumers holding one each
  const auto stage_of = [&](int c) { return 2 * swz_region_bytes(n, c * kTmaChunk, 2); };
  int nc_max = 1;
  for (int c = 3; c <= 255 && stage_of(c) <= kGramBudget / 9; c += 2) nc_max = c;
  const int64_t chunks = D / kTmaChunk;
  const int64_t ns0 = (chunks + nc_max - 1) / nc_max;
  int nc = static_cast<int>((chunks + ns0 - 1) / ns0);
  if (nc % 2 == 0) ++nc;  // <= nc_max, which is odd
  geo = WarpGeometry{};
  geo.tpi = 1;
  geo.sl = nc * kTmaChunk;
  geo.ns = static_cast<int>((D + geo.sl - 1) / geo.sl);
  geo.pitch = geo.sl;
  geo.stage_bytes = stage_of(nc);
  if (!ring_stage(geo, kBigRingWarps, T, sm_count(), kSwzAlign, kGramBudget)) return false;
  geo.consumers = std::min(geo.consumers, kBigRingWarps - 1);
  prefer_producers(geo);
  geo.wait_limit = wait_poll_limit();
  geo.gram_mma = kGramSwizzled;
  return true;
}

template <typename T, typename P, int NMAX, bool PROJ>
int launch_big_bwd_ring_n(int n, const WarpGeometry& geo_in, const RingMaps& maps, const MixBwdArgs& a,
                          cudaStream_t s) {
  WarpGeometry geo = geo_in;
  geo.status = timeout_word(s);
  auto* k = big_bwd_ring_kernel<T, P, NMAX, PROJ>;
  if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;
  const dim3 block((geo.consumers + 1) * 32, 1, 1);
  if (int rc = launch_ring(k, geo.grid, block, geo.smem_bytes, s, a, geo, maps, n)) return rc;
  return launch_status();
}

// The ring kernel when the shape and the pointers allow it (returns
// HC_ERR_UNSUPPORTED_N otherwise, so the caller runs big_bwd_kernel).
template <typename T, typename P, bool PROJ>
int launch_big_bwd_ring(int n, const MixBwdArgs& a, cudaStream_t s) {
  if constexpr (sizeof(T) != 2) {
    return HC_ERR_UNSUPPORTED_N;
  } else {
    WarpGeometry geo;
    if (!HC_GRAM_MMA || !aligned16(a.g) || !aligned16(a.x) || (a.grad_x && !aligned4(a.grad_x)) ||
        !big_ring_geometry(geo, n, a.T, a.D))
      return HC_ERR_UNSUPPORTED_N;
    RingMaps maps{};
    const void* base[2] = {a.g, a.x};
    const int rows[2] = {n, n};
    if (!ring_tensor_maps_swz(geo, maps, base, rows, 2, a.T, a.D, 2)) return HC_ERR_UNSUPPORTED_N;
    geo.tma = 1;
    return n <= 16 ? launch_big_bwd_ring_n<T, P, 16, PROJ>(n, geo, maps, a, s)
                   : launch_big_bwd_ring_n<T, P, 32, PROJ>(n, geo, maps, a, s);
  }
}

template <typename T, typename P, int NMAX, bool PROJ>
int launch_big_fwd_ring_n(int n, const WarpGeometry& geo_in, const RingMaps& maps, const MixFwdArgs& a,
                          cudaStream_t s) {
  WarpGeometry geo = geo_in;
  geo.status = timeout_word(s);
  auto* k = big_fwd_ring_kernel<T, P, NMAX, PROJ>;
  if (int rc = warp_prepare(k, geo.smem_bytes)) return rc;
  const dim3 block((geo.consumers + 1) * 32, 1, 1);
  if (int rc = launch_ring(k, geo.grid, block, geo.smem_bytes, s, a, geo, maps, n)) return rc;
  return launch_status();
}

// The forward ring kernel when the shape and the pointers allow it (returns
// HC_ERR_UNSUPPORTED_N otherwise, so the caller runs big_fwd_kernel).
template <typename T, typename P, bool PROJ>
int launch_big_fwd_ring(int n, const MixFwdArgs& a, cudaStream_t s) {
  if constexpr (sizeof(T) != 2) {
    return HC_ERR_UNSUPPORTED_N;
  } else {
    WarpGeometry geo;
    if (!HC_GRAM_MMA || !aligned16(a.x) || !aligned16(a.src) || !aligned4(a.out) ||
        !big_ring_geometry(geo, n, a.T, a.D))
      return HC_ERR_UNSUPPORTED_N;
    RingMaps maps{};
    const void* base[2] = {a.x, a.src};
    const int rows[2] = {n, n};
    if (!ring_tensor_maps_swz(geo, maps, base, rows, 2, a.T, a.D, 2)) return HC_ERR_UNSUPPORTED_N;
    geo.tma = 1;
    return n <= 16 ? launch_big_fwd_ring_n<T, P, 16, PROJ>(n, geo, maps, a, s)
                   : launch_big_fwd_ring_n<T, P, 32, PROJ>(n, geo, maps, a, s);
  }
}

}  // namespace hc
