// generator.cuh — per-token assembly of CGHC's generator A (n <= 8), forward
// and backward, float32, as device functions of one thread per token with
// everything in registers (generator.cu launches them alone; expm.cu fuses
// them with the Pade matrix exponential).
//
// Reference: hyperconnections/cghc.py:219-315 (compute_generator). With the
// module's pre-activations given per token
//   M      = conserv_A + conv_pred(x)              [n, n]  (conservative)
//   lc     = log_dt_conserv + dt_proj_conserv(x)   [n_dt]
//   ld     = log_dt_diss + dt_proj_diss(x)         [n_dt]
//   R      = diss_A + diss_pred(x)                 [n, n]  (PSD dissipation)
//   dpre   = diss_diag + diss_pred(x)              [n]     (diagonal dissipation)
//   S      = laplacian_A + laplacian_pred(x)       [n, n]  (graph Laplacian)
// and n_dt = n (vec_dt) or 1:
//   dt_c = lo_c + (hi_c - lo_c) sigmoid(lc),  dt_d = lo_d + (hi_d - lo_d) sigmoid(ld)
//   A  =  W(dt_c) (M - M^T)                                       conservative
//       - W(dt_d) (R R^T / sqrt(n))                                PSD
//       - diag(dt_d * softplus(dpre))                              diagonal
//       - W(dt_d) (diag(rowsum(adj)) - adj),                       Laplacian
//         adj = softplus((S + S^T) / 2) with a zero diagonal
// where W(dt) X = dt X for a scalar dt and sqrt(dt_i) X_ij sqrt(dt_j) per
// stream (the sandwich of cghc.py:245-251). softplus has PyTorch's default
// threshold (x > 20: x). The backward is reverse mode through the same steps.
#pragma once

#include "common.cuh"

namespace hc {
namespace {

constexpr int kGenThreads = 128;
enum : int { kConserv = 1, kPsd = 2, kDiag = 4, kLap = 8 };

struct GenArgs {
  const float* M;
  const float* lc;
  const float* ld;
  const float* R;
  const float* dpre;
  const float* S;
  const float* G;   // backward: dL/dA
  float* A;         // forward output
  float* dM;
  float* dlc;
  float* dld;
  float* dR;
  float* ddpre;
  float* dS;
  int64_t T;
  float lo_c, hi_c, lo_d, hi_d;
};

__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float softplusf(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus_grad(float x) { return x > 20.f ? 1.f : sigmoidf(x); }

// dt per stream (vec) or one scalar broadcast to all streams.
template <int N, bool VEC>
__device__ __forceinline__ void dt_of(const float* logit, int64_t t, float lo, float hi, float* dt, float* sg) {
  if constexpr (VEC) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      sg[i] = sigmoidf(logit[t * N + i]);
      dt[i] = lo + (hi - lo) * sg[i];
    }
  } else {
    const float s = sigmoidf(logit[t]);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      sg[i] = s;
      dt[i] = lo + (hi - lo) * s;
    }
  }
}

// W(dt) X: scalar dt * X, or sqrt(dt_i) X_ij sqrt(dt_j).
template <int N, bool VEC>
__device__ __forceinline__ float wscale(const float* dt, const float* sq, int i, int j) {
  if constexpr (VEC) {
    return sq[i] * sq[j];
  } else {
    return dt[0];
  }
}

template <int N, bool VEC>
__device__ void gen_forward_token(const GenArgs& a, int flags, int64_t t, float* A) {
  const float inv_sqrt_n = rsqrtf(static_cast<float>(N));
#pragma unroll
  for (int k = 0; k < N * N; ++k) A[k] = 0.f;
  if (flags & kConserv) {
    float dt[N], sg[N], sq[N], m[N * N];
    dt_of<N, VEC>(a.lc, t, a.lo_c, a.hi_c, dt, sg);
#pragma unroll
    for (int i = 0; i < N; ++i) sq[i] = sqrtf(dt[i]);
#pragma unroll
    for (int k = 0; k < N * N; ++k) m[k] = a.M[t * N * N + k];
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) A[i * N + j] += wscale<N, VEC>(dt, sq, i, j) * (m[i * N + j] - m[j * N + i]);
  }
  if (flags & (kPsd | kDiag | kLap)) {
    float dt[N], sg[N], sq[N];
    dt_of<N, VEC>(a.ld, t, a.lo_d, a.hi_d, dt, sg);
#pragma unroll
    for (int i = 0; i < N; ++i) sq[i] = sqrtf(dt[i]);
    if (flags & kPsd) {
      float r[N * N];
#pragma unroll
      for (int k = 0; k < N * N; ++k) r[k] = a.R[t * N * N + k];
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float kij = 0.f;
#pragma unroll
          for (int l = 0; l < N; ++l) kij = fmaf(r[i * N + l], r[j * N + l], kij);
          A[i * N + j] -= wscale<N, VEC>(dt, sq, i, j) * (kij * inv_sqrt_n);
        }
    }
    if (flags & kDiag) {
#pragma unroll
      for (int i = 0; i < N; ++i) A[i * N + i] -= dt[i] * softplusf(a.dpre[t * N + i]);
    }
    if (flags & kLap) {
      float adj[N * N], deg[N];
#pragma unroll
      for (int i = 0; i < N; ++i) {
        deg[i] = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float sij = 0.5f * (a.S[t * N * N + i * N + j] + a.S[t * N * N + j * N + i]);
          adj[i * N + j] = i == j ? 0.f : softplusf(sij);
        }
#pragma unroll
        for (int j = 0; j < N; ++j) deg[i] += adj[i * N + j];
      }
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float lij = (i == j ? deg[i] : 0.f) - adj[i * N + j];
          A[i * N + j] -= wscale<N, VEC>(dt, sq, i, j) * lij;
        }
    }
  }
}

// Reverse mode of W(dt) X for one term: adds dL/dX into dX and dL/d(dt) into
// ddt, given the term's upstream gradient sign * G.
template <int N, bool VEC>
__device__ __forceinline__ void wscale_bwd(const float* G, float sign, const float* X, const float* dt,
                                           const float* sq, float* dX, float* ddt) {
  if constexpr (VEC) {
    // P_ij = sq_i X_ij sq_j: dX_ij = g_ij sq_i sq_j; dsq_i = sum_j g_ij X_ij sq_j + sum_j g_ji X_ji sq_j
    float dsq[N];
#pragma unroll
    for (int i = 0; i < N; ++i) dsq[i] = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float g = sign * G[i * N + j];
        dX[i * N + j] += g * sq[i] * sq[j];
        dsq[i] += g * X[i * N + j] * sq[j];
        dsq[j] += g * X[i * N + j] * sq[i];
      }
#pragma unroll
    for (int i = 0; i < N; ++i) ddt[i] += dsq[i] * 0.5f / sq[i];  // sq = sqrt(dt)
  } else {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const float g = sign * G[i * N + j];
        dX[i * N + j] += g * dt[0];
        s += g * X[i * N + j];
      }
    ddt[0] += s;
  }
}

// Reverse mode of gen_forward_token for token t, given G = dL/dA of that
// token: writes the gradients of the pre-activations that a asks for.
template <int N, bool VEC>
__device__ void gen_backward_token(const GenArgs& a, int flags, int64_t t, const float (&G)[N * N]) {
  constexpr int ND = VEC ? N : 1;
  const float inv_sqrt_n = rsqrtf(static_cast<float>(N));

  if (flags & kConserv) {
    float dt[N], sg[N], sq[N], m[N * N], skew[N * N], dskew[N * N], ddt[N];
    dt_of<N, VEC>(a.lc, t, a.lo_c, a.hi_c, dt, sg);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      sq[i] = sqrtf(dt[i]);
      ddt[i] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < N * N; ++k) m[k] = a.M[t * N * N + k];
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) {
        skew[i * N + j] = m[i * N + j] - m[j * N + i];
        dskew[i * N + j] = 0.f;
      }
    wscale_bwd<N, VEC>(G, 1.f, skew, dt, sq, dskew, ddt);
    if (a.dM) {
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) a.dM[t * N * N + i * N + j] = dskew[i * N + j] - dskew[j * N + i];
    }
    if (a.dlc) {
#pragma unroll
      for (int i = 0; i < ND; ++i) a.dlc[t * ND + i] = ddt[i] * (a.hi_c - a.lo_c) * sg[i] * (1.f - sg[i]);
    }
  }
  if (flags & (kPsd | kDiag | kLap)) {
    float dt[N], sg[N], sq[N], ddt[N];
    dt_of<N, VEC>(a.ld, t, a.lo_d, a.hi_d, dt, sg);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      sq[i] = sqrtf(dt[i]);
      ddt[i] = 0.f;
    }
    if (flags & kPsd) {
      float r[N * N], K[N * N], dK[N * N];
#pragma unroll
      for (int k = 0; k < N * N; ++k) {
        r[k] = a.R[t * N * N + k];
        dK[k] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) {
          float kij = 0.f;
#pragma unroll
          for (int l = 0; l < N; ++l) kij = fmaf(r[i * N + l], r[j * N + l], kij);
          K[i * N + j] = kij * inv_sqrt_n;
        }
      wscale_bwd<N, VEC>(G, -1.f, K, dt, sq, dK, ddt);
      if (a.dR) {  // K = R R^T / sqrt(n): dR = (dK + dK^T) R / sqrt(n)
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int l = 0; l < N; ++l) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < N; ++j) s = fmaf(dK[i * N + j] + dK[j * N + i], r[j * N + l], s);
            a.dR[t * N * N + i * N + l] = s * inv_sqrt_n;
          }
      }
    }
    if (flags & kDiag) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float x = a.dpre[t * N + i];
        const float g = -G[i * N + i];
        ddt[VEC ? i : 0] += g * softplusf(x);
        if (a.ddpre) a.ddpre[t * N + i] = g * dt[i] * softplus_grad(x);
      }
    }
    if (flags & kLap) {
      float sym[N * N], L[N * N], dL[N * N];
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) {
          sym[i * N + j] = 0.5f * (a.S[t * N * N + i * N + j] + a.S[t * N * N + j * N + i]);
          dL[i * N + j] = 0.f;
        }
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float deg = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) deg += i == j ? 0.f : softplusf(sym[i * N + j]);
#pragma unroll
        for (int j = 0; j < N; ++j) L[i * N + j] = i == j ? deg : -softplusf(sym[i * N + j]);
      }
      wscale_bwd<N, VEC>(G, -1.f, L, dt, sq, dL, ddt);
      if (a.dS) {
        // L = diag(rowsum(adj)) - adj: d adj_ij = dL_ii - dL_ij (i != j);
        // adj = softplus(sym), zero diagonal; sym = (S + S^T) / 2
        float dsym[N * N];
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = 0; j < N; ++j)
            dsym[i * N + j] = i == j ? 0.f : (dL[i * N + i] - dL[i * N + j]) * softplus_grad(sym[i * N + j]);
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = 0; j < N; ++j) a.dS[t * N * N + i * N + j] = 0.5f * (dsym[i * N + j] + dsym[j * N + i]);
      }
    }
    if (a.dld) {  // with a scalar dt every term accumulated into ddt[0]
#pragma unroll
      for (int i = 0; i < ND; ++i) a.dld[t * ND + i] = ddt[i] * (a.hi_d - a.lo_d) * sg[i] * (1.f - sg[i]);
    }
  }
}

// Host-side argument check of the generator entry points.
int check_gen(const GenArgs& a, int n, int flags) {
  if (a.T < 0 || a.T > (int64_t(1) << 37)) return HC_ERR_BAD_SIZE;
  if (n < 1 || n > 8) return HC_ERR_UNSUPPORTED_N;
  if (flags <= 0 || flags > 15) return HC_ERR_BAD_SIZE;
  if (a.T == 0) return HC_OK;
  if ((flags & kConserv) && (!a.M || !a.lc)) return HC_ERR_NULL_POINTER;
  if ((flags & (kPsd | kDiag | kLap)) && !a.ld) return HC_ERR_NULL_POINTER;
  if ((flags & kPsd) && !a.R) return HC_ERR_NULL_POINTER;
  if ((flags & kDiag) && !a.dpre) return HC_ERR_NULL_POINTER;
  if ((flags & kLap) && !a.S) return HC_ERR_NULL_POINTER;
  const void* ptrs[] = {a.M, a.lc, a.ld, a.R, a.dpre, a.S, a.G, a.A, a.dM, a.dlc, a.dld, a.dR, a.ddpre, a.dS};
  for (const void* p : ptrs)
    if (p && !aligned4(p)) return HC_ERR_ALIGNMENT;
  return HC_OK;
}

}  // namespace
}  // namespace hc
