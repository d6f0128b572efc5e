// bign.cuh — stream_mix_add for 9 <= n <= 32 streams (forward and backward).
//
// Same arithmetic as the n <= 8 kernels (reference ops/stream_mix_small_nb.py
// and stream_mix_big_nb.py, the latter dispatched for N >= 16):
//   out_i = sum_j Phi_ij x_j [+ c_i (v^T x)] + Y_i,          c = v - Phi v
//   grad_x_j = sum_i Phi_ij G_i [+ v_j (c^T G)]
//   grad_Phi_ij = sum_d G_i (x_j - v_j v^T x)
//   grad_v = rho - Phi^T rho + sum_d (c^T G) x,  rho_i = sum_d G_i (v^T x)
//
// An n x n matrix no longer fits a lane's registers, so the layout changes:
// one CTA per token; Phi, v and c live in shared memory and are read as
// broadcasts.
//   forward   each thread holds the column of x at its elements (n values per
//             element, one 32-bit word of the stream per row) and produces the
//             n outputs row by row: every byte of x, Y and out crosses HBM once.
//   backward  the token is staged in slices of D as fp32 rows in shared
//             memory, augmented with one extra row each: c^T G below the G
//             rows and v^T x below the x rows (projection only). grad_x is
//             Phi^T G per element column; the parameter gradients are the Gram
//             matrix M = G_aug X_aug^T summed over D: M[:n,:n] = sum G x^T,
//             M[i,n] = rho_i, M[n,j] = sum (c^T G) x_j, so
//             grad_Phi = M[:n,:n] - rho v^T and grad_v follow without a second
//             pass. The Gram runs in 4 x 4 register tiles, several threads per
//             tile over disjoint elements, folded once at the end.
#pragma once

#include "mix_warp.cuh"

namespace hc {

constexpr int kBigThreads = 256;
constexpr int kBigMaxN = 32;

// One thread's group of consecutive elements: one 32-bit word of the stream
// (2 elements for 16-bit types, 1 for fp32) when rows are word-aligned, else 1.
template <typename T, bool VEC>
struct BigIO {
  static constexpr int K = VEC ? Word<T>::K : 1;
  __device__ static __forceinline__ void load(const T* p, float* f) {
    if constexpr (VEC) {
      Word<T>::get(__ldg(reinterpret_cast<const unsigned int*>(p)), f);
    } else {
      f[0] = Elem<T>::to_f(p[0]);
    }
  }
  __device__ static __forceinline__ void store(T* p, const float* f) {
    if constexpr (VEC) {
      *reinterpret_cast<uint32_t*>(p) = Word<T>::put(f);
    } else {
      p[0] = Elem<T>::from_f(f[0]);
    }
  }
};

// Phi, v and c = v - Phi v of token t into shared memory, zero-padded to
// NMAX so that rows can be read as float4 without bounds: phi[i*NMAX + j]
// (TRANS: phi[j*NMAX + i]).
template <typename P, int NMAX, bool PROJ, bool TRANS>
__device__ __forceinline__ void big_params(const void* phi_p, const void* v_p, int64_t t, int n, float* phi,
                                           float* vv, float* cc) {
  const P* ph = static_cast<const P*>(phi_p) + t * n * n;
  for (int k = threadIdx.x; k < NMAX * NMAX; k += blockDim.x) {
    const int i = k / NMAX, j = k % NMAX;
    const float val = (i < n && j < n) ? Elem<P>::to_f(ph[i * n + j]) : 0.f;
    phi[TRANS ? j * NMAX + i : k] = val;
  }
  if (threadIdx.x < NMAX) {
    vv[threadIdx.x] = (PROJ && threadIdx.x < n) ? Elem<P>::to_f(static_cast<const P*>(v_p)[t * n + threadIdx.x]) : 0.f;
    cc[threadIdx.x] = 0.f;
  }
  __syncthreads();
  if constexpr (PROJ) {
    if (threadIdx.x < n) {
      const int i = threadIdx.x;
      float hv = 0.f;
      for (int j = 0; j < n; ++j) hv = fmaf(phi[TRANS ? j * NMAX + i : i * NMAX + j], vv[j], hv);
      cc[i] = vv[i] - hv;
    }
    __syncthreads();
  }
}

template <typename T, typename P, int NMAX, bool PROJ, bool VEC>
__global__ void __launch_bounds__(kBigThreads) big_fwd_kernel(const MixFwdArgs a, int n) {
  using IO = BigIO<T, VEC>;
  constexpr int K = IO::K;
  __shared__ __align__(16) float phi[NMAX * NMAX];
  __shared__ float vv[NMAX], cc[NMAX];
  const int64_t t = blockIdx.x;
  big_params<P, NMAX, PROJ, false>(a.phi, a.v, t, n, phi, vv, cc);
  const int64_t D = a.D;
  const T* xt = static_cast<const T*>(a.x) + t * n * D;
  const T* yt = static_cast<const T*>(a.src) + t * n * D;
  T* ot = static_cast<T*>(a.out) + t * n * D;
  for (int64_t e = static_cast<int64_t>(threadIdx.x) * K; e < D; e += static_cast<int64_t>(blockDim.x) * K) {
    float xe[NMAX][K];  // rows >= n stay zero and meet zero padding in phi
#pragma unroll
    for (int j = 0; j < NMAX; ++j) {
      if (j < n) {
        IO::load(xt + j * D + e, xe[j]);
      } else {
#pragma unroll
        for (int k = 0; k < K; ++k) xe[j][k] = 0.f;
      }
    }
    float s[K];
    if constexpr (PROJ) {
#pragma unroll
      for (int k = 0; k < K; ++k) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < NMAX; ++j) acc = fmaf(vv[j], xe[j][k], acc);
        s[k] = acc;
      }
    }
    // output rows in groups of 4; the next group's Y rows are requested
    // before this group's arithmetic, so several loads per warp are in flight
    constexpr int RG = 4;
    float ya[RG][K], yb[RG][K];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      if (r < n) IO::load(yt + r * D + e, ya[r]);
    }
    for (int g0 = 0; g0 < n; g0 += RG) {
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        if (g0 + RG + r < n) IO::load(yt + (g0 + RG + r) * D + e, yb[r]);
      }
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const int i = g0 + r;
        if (i < n) {
          float o[K];
#pragma unroll
          for (int k = 0; k < K; ++k) o[k] = 0.f;
          const float4* prow = reinterpret_cast<const float4*>(phi + i * NMAX);
#pragma unroll
          for (int q = 0; q < NMAX / 4; ++q) {
            const float4 p4 = prow[q];
#pragma unroll
            for (int k = 0; k < K; ++k) {
              o[k] = fmaf(p4.x, xe[4 * q][k], o[k]);
              o[k] = fmaf(p4.y, xe[4 * q + 1][k], o[k]);
              o[k] = fmaf(p4.z, xe[4 * q + 2][k], o[k]);
              o[k] = fmaf(p4.w, xe[4 * q + 3][k], o[k]);
            }
          }
#pragma unroll
          for (int k = 0; k < K; ++k) {
            if constexpr (PROJ) o[k] = fmaf(cc[i], s[k], o[k]);
            o[k] = o[k] + ya[r][k];
          }
          IO::store(ot + i * D + e, o);
        }
      }
#pragma unroll
      for (int r = 0; r < RG; ++r)
#pragma unroll
        for (int k = 0; k < K; ++k) ya[r][k] = yb[r][k];
    }
  }
}

// Backward geometry: slice length of the staged rows, its row pitch (padded
// against bank conflicts between rows) and the Gram tiling.
template <int NMAX> struct BigBwd {
  static constexpr int SL = 256;                      // elements per staged slice
  static constexpr int EPT = SL / kBigThreads;        // elements per thread per row
  static constexpr int PITCH = SL + 4;
  static constexpr int ROWS = NMAX + 4;               // n + augmented row, padded to a tile multiple
};

// Dynamic shared memory of the backward: staged G and x rows (fp32), then
// Phi^T, v, c and the folded Gram.
template <int NMAX>
constexpr size_t big_bwd_smem() {
  using B = BigBwd<NMAX>;
  const size_t stage = 2ull * B::ROWS * B::PITCH;
  const size_t fold = static_cast<size_t>(kBigThreads) * 16;
  return ((stage > fold ? stage : fold) + NMAX * NMAX + 2 * NMAX + B::ROWS * B::ROWS) * sizeof(float);
}

template <typename T, typename P, int NMAX, bool PROJ, bool VEC>
__global__ void __launch_bounds__(kBigThreads) big_bwd_kernel(const MixBwdArgs a, int n) {
  using B = BigBwd<NMAX>;
  constexpr int SL = B::SL, EPT = B::EPT, PITCH = B::PITCH, ROWS = B::ROWS;
  extern __shared__ __align__(16) float bsm[];
  float* gs = bsm;                  // [ROWS][PITCH]  G rows, row n = c^T G (projection)
  float* xs = bsm + ROWS * PITCH;   // [ROWS][PITCH]  x rows, row n = v^T x (projection)
  const size_t stage = 2ull * ROWS * PITCH;
  const size_t fold = static_cast<size_t>(kBigThreads) * 16;
  float* phiT = bsm + (stage > fold ? stage : fold);  // [NMAX][NMAX], phiT[j][i] = Phi_ij
  float* vv = phiT + NMAX * NMAX;
  float* cc = vv + NMAX;
  float* gram = cc + NMAX;          // [ROWS][ROWS]
  const int64_t t = blockIdx.x;
  big_params<P, NMAX, PROJ, true>(a.phi, a.v, t, n, phiT, vv, cc);

  const int na = n + (PROJ ? 1 : 0);   // rows of the augmented Gram
  const int np = (na + 3) & ~3;        // padded to whole 4 x 4 tiles
  const int tpd = np / 4;
  const int ntiles = tpd * tpd;
  const int dparts = kBigThreads / ntiles;
  const int tid = threadIdx.x;
  const bool gram_thread = tid < ntiles * dparts;
  const int tile = gram_thread ? tid / dparts : 0;
  const int dp = gram_thread ? tid % dparts : 0;
  const int ti = (tile / tpd) * 4, tj = (tile % tpd) * 4;
  float acc[4][4];
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[p][q] = 0.f;

  // rows NMAX..ROWS-1 stay zero for the whole kernel (rows n..NMAX-1 are
  // rewritten with zeros every slice)
  for (int k = tid; k < (ROWS - NMAX) * PITCH; k += blockDim.x) {
    gs[NMAX * PITCH + k] = 0.f;
    xs[NMAX * PITCH + k] = 0.f;
  }

  const int64_t D = a.D;
  const T* gt = static_cast<const T*>(a.g) + t * n * D;
  const T* xt = static_cast<const T*>(a.x) + t * n * D;
  T* gxt = a.grad_x ? static_cast<T*>(a.grad_x) + t * n * D : nullptr;
  for (int64_t d0 = 0; d0 < D; d0 += SL) {
    const int len = static_cast<int>(D - d0 < SL ? D - d0 : SL);
    // this thread's elements of every row, all loads in flight together
    float gr[NMAX][EPT], xr[NMAX][EPT];
#pragma unroll
    for (int r = 0; r < NMAX; ++r) {
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        const int e = tid + k * kBigThreads;
        const bool ok = r < n && e < len;
        gr[r][k] = ok ? Elem<T>::to_f(gt[r * D + d0 + e]) : 0.f;
        xr[r][k] = ok ? Elem<T>::to_f(xt[r * D + d0 + e]) : 0.f;
      }
    }
    float bt[EPT], sv[EPT];
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      float b = 0.f, sa = 0.f;
      if constexpr (PROJ) {
#pragma unroll
        for (int r = 0; r < NMAX; ++r) {
          b = fmaf(cc[r], gr[r][k], b);
          sa = fmaf(vv[r], xr[r][k], sa);
        }
      }
      bt[k] = b;
      sv[k] = sa;
    }
    // grad_x = Phi^T G [+ v (c^T G)] straight from the registers
    if (gxt) {
      for (int j = 0; j < n; ++j) {
        float o[EPT];
#pragma unroll
        for (int k = 0; k < EPT; ++k) o[k] = 0.f;
        const float4* pcol = reinterpret_cast<const float4*>(phiT + j * NMAX);
#pragma unroll
        for (int q = 0; q < NMAX / 4; ++q) {
          const float4 p4 = pcol[q];
#pragma unroll
          for (int k = 0; k < EPT; ++k) {
            o[k] = fmaf(p4.x, gr[4 * q][k], o[k]);
            o[k] = fmaf(p4.y, gr[4 * q + 1][k], o[k]);
            o[k] = fmaf(p4.z, gr[4 * q + 2][k], o[k]);
            o[k] = fmaf(p4.w, gr[4 * q + 3][k], o[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < EPT; ++k) {
          const int e = tid + k * kBigThreads;
          if (e < len) {
            float val = o[k];
            if constexpr (PROJ) val = fmaf(vv[j], bt[k], val);
            gxt[j * D + d0 + e] = Elem<T>::from_f(val);
          }
        }
      }
    }
    __syncthreads();  // the previous slice's Gram reads are done
#pragma unroll
    for (int r = 0; r < NMAX; ++r) {
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        gs[r * PITCH + tid + k * kBigThreads] = gr[r][k];
        xs[r * PITCH + tid + k * kBigThreads] = xr[r][k];
      }
    }
    if constexpr (PROJ) {
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        gs[n * PITCH + tid + k * kBigThreads] = bt[k];
        xs[n * PITCH + tid + k * kBigThreads] = sv[k];
      }
    }
    __syncthreads();
    // Gram tiles over this slice, four consecutive elements per step
    if (gram_thread) {
      for (int e = dp * 4; e < SL; e += dparts * 4) {
        float4 ga[4], xb[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          ga[p] = *reinterpret_cast<const float4*>(gs + (ti + p) * PITCH + e);
          xb[p] = *reinterpret_cast<const float4*>(xs + (tj + p) * PITCH + e);
        }
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[p][q] = fmaf(ga[p].x, xb[q].x, acc[p][q]);
            acc[p][q] = fmaf(ga[p].y, xb[q].y, acc[p][q]);
            acc[p][q] = fmaf(ga[p].z, xb[q].z, acc[p][q]);
            acc[p][q] = fmaf(ga[p].w, xb[q].w, acc[p][q]);
          }
      }
    }
  }
  // fold the partial tiles (the stage area is free once every thread is past its Gram)
  __syncthreads();
  float* red = bsm;
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int q = 0; q < 4; ++q) red[tid * 16 + p * 4 + q] = gram_thread ? acc[p][q] : 0.f;
  __syncthreads();
  for (int k = tid; k < na * na; k += blockDim.x) {
    const int i = k / na, j = k % na;
    const int tl = (i / 4) * tpd + j / 4;
    float s = 0.f;
    for (int q = 0; q < dparts; ++q) s += red[(tl * dparts + q) * 16 + (i % 4) * 4 + (j % 4)];
    gram[i * ROWS + j] = s;
  }
  __syncthreads();
  if (a.grad_phi) {
    for (int k = tid; k < n * n; k += blockDim.x) {
      const int i = k / n, j = k % n;
      float gpv = gram[i * ROWS + j];
      if constexpr (PROJ) gpv = gpv - vv[j] * gram[i * ROWS + n];  // - rho_i v_j
      a.grad_phi[t * n * n + k] = gpv;
    }
  }
  if constexpr (PROJ) {
    if (a.grad_v && tid < n) {
      const int j = tid;
      float ht = 0.f;
      for (int i = 0; i < n; ++i) ht = fmaf(phiT[j * NMAX + i], gram[i * ROWS + n], ht);
      a.grad_v[t * n + j] = (gram[j * ROWS + n] - ht) + gram[n * ROWS + j];
    }
  }
}

template <typename T, typename P, bool PROJ, bool VEC>
int launch_big_fwd(int n, const MixFwdArgs& a, cudaStream_t s) {
  const unsigned grid = static_cast<unsigned>(a.T);
  if (n <= 16) {
    big_fwd_kernel<T, P, 16, PROJ, VEC><<<grid, kBigThreads, 0, s>>>(a, n);
  } else {
    big_fwd_kernel<T, P, 32, PROJ, VEC><<<grid, kBigThreads, 0, s>>>(a, n);
  }
  return launch_status();
}

template <typename T, typename P, bool PROJ, bool VEC, int NMAX>
int launch_big_bwd_n(int n, const MixBwdArgs& a, cudaStream_t s) {
  auto* k = big_bwd_kernel<T, P, NMAX, PROJ, VEC>;
  constexpr int smem = static_cast<int>(big_bwd_smem<NMAX>());
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return HC_ERR_LAUNCH;
  k<<<static_cast<unsigned>(a.T), kBigThreads, smem, s>>>(a, n);
  return launch_status();
}

template <typename T, typename P, bool PROJ, bool VEC>
int launch_big_bwd(int n, const MixBwdArgs& a, cudaStream_t s) {
  return n <= 16 ? launch_big_bwd_n<T, P, PROJ, VEC, 16>(n, a, s) : launch_big_bwd_n<T, P, PROJ, VEC, 32>(n, a, s);
}

// Per-dtype entry points (bign_<dtype>.cu): vec = 32-bit word access.
#define HC_DECLARE_BIG(SFX)                                                                                 \
  int big_fwd_##SFX(bool proj, bool vec, bool param_is_f32, int n, const MixFwdArgs& a, cudaStream_t s);    \
  int big_bwd_##SFX(bool proj, bool vec, bool param_is_f32, int n, const MixBwdArgs& a, cudaStream_t s);
HC_DECLARE_BIG(f32)
HC_DECLARE_BIG(f16)
HC_DECLARE_BIG(bf16)
#undef HC_DECLARE_BIG

}  // namespace hc
