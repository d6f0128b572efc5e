/*
 * hcops.h — C ABI of libhcops.so, the sm_100a kernels of the hyper-connections
 * hot path (batched small-matrix exponential and fused stream mixing).
 *
 * Every entry point:
 *   - takes DEVICE pointers, element counts and a cudaStream_t passed as void*
 *     (NULL = legacy default stream);
 *   - enqueues its kernels on that stream and returns without synchronising;
 *   - allocates no device memory (scratch memory, where a path needs it, is
 *     passed in by the caller) and keeps no per-call state;
 *   - returns HC_OK (0) or one of the HC_ERR_* codes below; hc_error_string()
 *     turns a code into text.
 * Process-wide state is limited to the status of bounded waits (below) and
 * the two hc_debug_* knobs.
 *
 * Bounded waits. Kernels that wait on each other's work (the bulk-copy ring
 * of the stream-mixing kernels, the grid barrier of the cooperative expm
 * forward) poll a bounded number of times. A wait that gives up leaves that
 * launch's outputs incomplete; the kernel records it in one word of pinned,
 * device-mapped host memory, and from then on every entry point that launches
 * work returns HC_ERR_TIMEOUT without launching, until hc_wait_timeouts(..., 1)
 * clears it (like a sticky CUDA error, the call after the failing one reports
 * it). The word is mapped (cudaHostAlloc, 64 bytes, once per process) at the
 * first launch of such a kernel on a stream that is not capturing a graph;
 * make one call of each op before capturing it.
 *
 * Layouts are dense row-major with the token (batch) index outermost:
 *   streams  x, Y, out, grad_out, grad_x   [T, n, D]   stream dtype
 *   layer output f, read output u           [T, D]      stream dtype
 *   mixing matrix Phi / H                   [T, n, n]   param dtype
 *   projection direction v                  [T, n]      param dtype
 *   read weights alpha, write weights beta  [T, n]      float32
 *   matrices for expm A, E, G, dA           [batch, n, n] float32
 *   m-block read / write: R [T,m,n], W [T,n,m] float32; f, u [T,m,D] stream dtype
 * All gradients of per-token parameters are written as float32.
 *
 * Citations name the reference interface each entry point replaces
 * (pjjajal/hyperconnections, paths relative to the project root).
 */
#ifndef HCOPS_H
#define HCOPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define HC_OK                 0
#define HC_ERR_NULL_POINTER   1  /* a required pointer is NULL                     */
#define HC_ERR_BAD_SIZE       2  /* negative size, or n / D out of range           */
#define HC_ERR_UNSUPPORTED_N  3  /* n (or m) outside the entry point's range      */
#define HC_ERR_DTYPE          4  /* unknown dtype code or unsupported combination  */
#define HC_ERR_ALIGNMENT      5  /* a float32 pointer is not 4-byte aligned        */
#define HC_ERR_SCRATCH        6  /* scratch buffer missing or too small            */
#define HC_ERR_LAUNCH         7  /* the CUDA launch itself failed                  */
#define HC_ERR_TIMEOUT        8  /* a bounded wait in an earlier launch gave up    */

/* ---- dtype codes ---------------------------------------------------------- */
#define HC_DTYPE_F32   0
#define HC_DTYPE_F16   1
#define HC_DTYPE_BF16  2

/* Text for a status code (static storage). */
const char* hc_error_string(int code);

/* Library ABI version; bumped whenever a signature below changes or an entry
 * point is added. */
int hc_abi_version(void);

/* Diagnostics: synchronises the current device, then stores in *count how
 * many bounded waits inside the kernels gave up since the last reset (0 in a
 * healthy run; a kernel that gives up leaves its outputs incomplete and
 * returns instead of spinning). reset != 0 clears the counters and the status
 * word, after which the entry points launch again. No reference counterpart
 * (the reference's Triton kernels have no such waits). */
int hc_wait_timeouts(unsigned int* count, int reset);

/* Non-blocking: the give-ups recorded in the status word so far (by kernels
 * that have reached their give-up; no synchronisation, so a launch still
 * running is not counted yet). 0 when no kernel with bounded waits has been
 * launched. No reference counterpart. */
int hc_timeout_status(unsigned int* count);

/* DEBUG / BENCHMARK HOOK, process-wide and read at every launch: overrides
 * the ring geometry of the pipelined stream-mixing kernels (target bytes of
 * one item, stages, consumer warps, producer lanes of the fill warp; 0 keeps
 * the automatic choice). Results do
 * not depend on these settings; a launch on another thread sees either the
 * old or the new values. Not for production use. No reference counterpart
 * (the reference autotunes its Triton block sizes,
 * ops/stream_mix_small_nb.py:52-67). */
int hc_debug_set_mix_tuning(int stage_bytes, int stages, int warps, int producers);

/* DEBUG / TEST HOOK, process-wide: the number of polls after which a data
 * wait of the ring kernels and the grid barrier of the cooperative expm give
 * up (0 restores the default of 2^22 polls, about a quarter of a second).
 * Lowering it makes waits run out on purpose, to test the HC_ERR_TIMEOUT
 * path; the ring's exit drain keeps the default. No reference counterpart. */
int hc_debug_set_wait_limit(unsigned int polls);

/* DEBUG / TEST HOOK: the ring geometry that the pipelined kernels would take
 * for one op and shape, by the same host arithmetic the launches use (no
 * device work; usable without a GPU, where the SM count is taken as 148).
 * op: 0 the fused step, 1 stream_mix_add (n <= 32; above 8 the
 * half-precision tensor-core ring, the same for both directions), 2 read,
 * 3 mix-write; bwd
 * non-zero for the backward; m and proj as for the op (ignored where it has
 * none). Streams are taken as 16-byte aligned. Writes min(out_len, 12) ints:
 * [ring (1; 0 when the shape takes a non-ring kernel, and every other field
 * 0), stages, consumer warps, producer lanes, tokens per item, elements per
 * slice, slices per token, stage bytes, dynamic shared memory bytes, side
 * rows (1 when the backward's one-row tensors come by consumer copies),
 * tensor-core Gram stages (0 none, 1 padded, 2 swizzled), CTAs].
 * Honours hc_debug_set_mix_tuning. No reference counterpart. */
int hc_debug_ring_geometry(int op, int bwd, int n, int m, int proj, int64_t T,
                           int64_t D, int stream_dtype, int* out, int out_len);

/* ===========================================================================
 * Batched matrix exponential, n <= 8, float32.
 * ======================================================================== */

/* Number of float32 words of scratch that hc_expm_t18_fwd / hc_expm_t18_bwd
 * need in global-scaling mode for a batch of `batch` matrices of order n
 * (the per-block partial maxima of ||A||_1). Returns 0 in error cases. */
int64_t hc_expm_t18_scratch_words(int64_t batch, int n);

/* E = exp(A) by the optimised Taylor polynomial of degree 18 (Bader, Blanes
 * and Casas 2019) with scaling and squaring, theta_18 = 3.01.
 *   per_matrix == 0: ONE scaling exponent for the whole batch, taken from
 *     max_b ||A_b||_1, as the reference does; `scratch` must hold
 *     hc_expm_t18_scratch_words(batch, n) floats.
 *   per_matrix != 0: each matrix gets its own exponent; scratch may be NULL.
 * Replaces: hyperconnections/ops/expm.py:69-106 (expm_t18 forward). */
int hc_expm_t18_fwd(const float* A, float* E, int64_t batch, int n,
                    float* scratch, int64_t scratch_words, int per_matrix,
                    void* stream);

/* dA = L_exp18(A^T, G): the adjoint Frechet derivative of the same T18
 * approximant (same scaling exponent as the forward), i.e. the gradient of
 * sum(G * expm_t18(A)) with respect to A. per_matrix: 0 global scaling (the
 * partial maxima are recomputed into scratch), 1 per-matrix scaling, 2 global
 * scaling reusing the partial maxima that hc_expm_t18_fwd left in `scratch`
 * for this same A (saves one pass over A; the caller keeps scratch intact
 * between the two calls). Any other value returns HC_ERR_BAD_SIZE, and so
 * does a per_matrix other than 0 or 1 in hc_expm_t18_fwd.
 * Replaces: the autograd backward of hyperconnections/ops/expm.py:69-106. */
int hc_expm_t18_bwd(const float* A, const float* G, float* dA, int64_t batch,
                    int n, float* scratch, int64_t scratch_words,
                    int per_matrix, void* stream);

/* The same result as hc_expm_t18_fwd with per_matrix == 0, for callers that
 * cannot allocate device memory: a plugin or FFI caller that only receives
 * pointers from a host framework owning all device memory, or a loop that
 * must not call cudaMalloc because it can synchronise the device. The
 * caller passes A and E only; the scratch (the per-CTA partial maxima of
 * ||A||_1, at most 1024 floats) lives in a fixed 4 KB device array inside the
 * library, which every GPU that loads the library keeps until exit. Limits:
 * the same batch bound as the other expm entry points (2^34 matrices, else
 * HC_ERR_BAD_SIZE); every batch within it fits the array, since the norm pass
 * strides over the batch with at most 1024 blocks. The first call on a device
 * looks up the array's device address once (cudaGetSymbolAddress); make that
 * first call before any stream capture. All calls share the one array and it
 * keeps the last call's contents; every slot a call reads is written earlier
 * in the same call, so nothing needs clearing, but calls that overlap on the
 * GPU (for example on two streams at once) race on it.
 * No counterpart in the reference. */
int hc_expm_t18_fwd_noalloc(const float* A, float* E, int64_t batch, int n,
                            void* stream);

/* E = exp(A) by diagonal Pade [7/7] with per-matrix scaling and squaring
 * (Higham 2005, theta_7 = 3.925724783138660 for unit roundoff 2^-24) and an
 * in-register Gauss-Jordan solve with partial pivoting.
 * Replaces: torch.linalg.matrix_exp at hyperconnections/cghc.py:321. */
int hc_expm_pade_fwd(const float* A, float* E, int64_t batch, int n,
                     void* stream);

/* dA = L_exp(A^T, G) of the Pade approximant (Al-Mohy and Higham 2009).
 * Replaces: the autograd backward of torch.linalg.matrix_exp at
 * hyperconnections/cghc.py:321. */
int hc_expm_pade_bwd(const float* A, const float* G, float* dA, int64_t batch,
                     int n, void* stream);

/* Sinkhorn-Knopp projection of exp(H) onto the doubly stochastic matrices:
 * X = exp(H), then `iters` times: divide each row by its sum, then each
 * column by its sum. H, P [batch, n, n] float32; 0 <= iters <= 256.
 * Replaces: hyperconnections/mhc.py:97-102 (MHC._sinkhorn_knopp). */
int hc_sinkhorn_fwd(const float* H, float* P, int64_t batch, int n, int iters,
                    void* stream);

/* dH = gradient of sum(G * sinkhorn(H)) with respect to H, the reverse of
 * every normalisation step (the autograd backward of mhc.py:97-102). */
int hc_sinkhorn_bwd(const float* H, const float* G, float* dH, int64_t batch,
                    int n, int iters, void* stream);

/* CGHC's generator A per token, from the module's pre-activations (float32):
 *   M = conserv_A + conv_pred(x) [T,n,n], lc = log_dt_conserv + dt_proj_conserv(x)
 *   [T,n_dt], R = diss_A + diss_pred(x) [T,n,n], dpre = diss_diag + diss_pred(x)
 *   [T,n], S = laplacian_A + laplacian_pred(x) [T,n,n], ld = log_dt_diss +
 *   dt_proj_diss(x) [T,n_dt]; n_dt = n if vec_dt else 1.
 * flags: 1 conservative, 2 PSD, 4 diagonal, 8 Laplacian dissipation (the
 * seven generator types are the combinations the reference allows); inputs of
 * absent terms may be NULL. A [T,n,n].
 * Replaces: hyperconnections/cghc.py:219-315 (compute_generator) after its
 * Linear layers. */
int hc_cghc_generator_fwd(const float* M, const float* lc, const float* R,
                          const float* dpre, const float* S, const float* ld,
                          float* A, int64_t T, int n, int vec_dt, int flags,
                          float dt_min_c, float dt_max_c, float dt_min_d,
                          float dt_max_d, void* stream);

/* Given G = dL/dA [T,n,n]: the gradients with respect to each pre-activation
 * (same shapes as the inputs; any may be NULL to skip it). */
int hc_cghc_generator_bwd(const float* M, const float* lc, const float* R,
                          const float* dpre, const float* S, const float* ld,
                          const float* G, float* dM, float* dlc, float* dR,
                          float* ddpre, float* dS, float* dld, int64_t T, int n,
                          int vec_dt, int flags, float dt_min_c, float dt_max_c,
                          float dt_min_d, float dt_max_d, void* stream);

/* CGHC's transition Phi = exp(A) [T,n,n] straight from the pre-activations
 * of hc_cghc_generator_fwd (same arguments and flags): the generator and the
 * Pade [7/7] exponential of hc_expm_pade_fwd in one kernel, bit for bit the
 * result of the two calls, without A's round trip through memory.
 * Replaces: hyperconnections/cghc.py:219-321 (compute_generator, then
 * torch.linalg.matrix_exp in compute_transition). */
int hc_cghc_transition_fwd(const float* M, const float* lc, const float* R,
                           const float* dpre, const float* S, const float* ld,
                           float* Phi, int64_t T, int n, int vec_dt, int flags,
                           float dt_min_c, float dt_max_c, float dt_min_d,
                           float dt_max_d, void* stream);

/* Given G = dL/dPhi [T,n,n]: the gradients with respect to each
 * pre-activation, as hc_cghc_generator_bwd gives them for dL/dA (A is
 * assembled again inside the kernel; any output may be NULL).
 * Replaces the autograd backward of cghc.py:219-321. */
int hc_cghc_transition_bwd(const float* M, const float* lc, const float* R,
                           const float* dpre, const float* S, const float* ld,
                           const float* G, float* dM, float* dlc, float* dR,
                           float* ddpre, float* dS, float* dld, int64_t T,
                           int n, int vec_dt, int flags, float dt_min_c,
                           float dt_max_c, float dt_min_d, float dt_max_d,
                           void* stream);

/* ===========================================================================
 * stream_mix_add: out = Phi x + Y              (v == NULL)
 *                 out = Phi x + (v - Phi v)(v^T x) + Y   (v != NULL)
 * x, Y, out share stream_dtype; Phi and v share param_dtype, which must be
 * HC_DTYPE_F32 or equal to stream_dtype. fp32 accumulation.
 * ======================================================================== */

/* 1 <= n <= 32: n <= 8 runs the register kernels, 9..32 the shared-memory
 * kernels (one CTA per token). Other entry points keep n <= 8.
 * Replaces: hyperconnections/ops/stream_mix.py:57-86 (stream_mix_add) ->
 * stream_mix_small_nb.py:75-132 (_stream_mix_fwd) and
 * stream_mix_big_nb.py:74-146 (_stream_mix_fwd_big_nb). */
int hc_stream_mix_fwd(const void* Phi, const void* x, const void* Y,
                      const void* v, void* out, int64_t B, int n, int64_t D,
                      int stream_dtype, int param_dtype, void* stream);

/* Given G = dL/dout [B,n,D] (stream dtype):
 *   grad_x   = Phi^T G (+ v beta^T)            [B,n,D] stream dtype (nullable)
 *   grad_Phi = G x_eff^T                        [B,n,n] float32     (nullable)
 *   grad_v   = rho - Phi^T rho + beta-part      [B,n]   float32     (nullable;
 *              only with v != NULL)
 * where, with v: alpha = v^T x, c = v - Phi v, beta = c^T G, x_eff = x - v alpha.
 * grad_Y is G itself and is not produced here.
 * Replaces: stream_mix_small_nb.py:341-391 (_StreamMixFn.backward) with its
 * kernels :148-197 (_stream_mix_bwd_dx) and :213-263 (_stream_mix_bwd_dPhi). */
int hc_stream_mix_bwd(const void* G, const void* Phi, const void* x,
                      const void* v, void* grad_x, float* grad_Phi,
                      float* grad_v, int64_t B, int n, int64_t D,
                      int stream_dtype, int param_dtype, void* stream);

/* ===========================================================================
 * Fused hyper-connection step with one backbone block (m = 1):
 *   u      = sum_j alpha_j x_j                      (width-read)
 *   x_out_i = sum_j H_ij x_j + beta_i f             (residual mix + depth-write)
 * H, alpha, beta are float32; x, f, u, x_out share stream_dtype.
 * Replaces the composition hyperconnections/cghc.py:410 (read einsum),
 * :417 (write einsum) and :449 -> ops/stream_mix.py:57 (stream_mix_add),
 * without materialising the write-out Y.
 * ======================================================================== */
int hc_fused_fwd(const void* x, const void* f, const float* H,
                 const float* alpha, const float* beta, void* u, void* x_out,
                 int64_t T, int n, int64_t D, int stream_dtype, void* stream);

/* Given g_u = dL/du [T,D] and g_x = dL/dx_out [T,n,D]:
 *   grad_x_j   = sum_i H_ij g_x_i + alpha_j g_u      [T,n,D] (nullable)
 *   grad_f     = sum_i beta_i g_x_i                  [T,D]   (nullable)
 *   grad_H_ij  = sum_d g_x_i x_j                     [T,n,n] float32 (nullable)
 *   grad_alpha_j = sum_d g_u x_j                     [T,n]   float32 (nullable)
 *   grad_beta_i  = sum_d g_x_i f                     [T,n]   float32 (nullable)
 * Replaces the autograd backward of the same composition (einsum backward at
 * cghc.py:410/:417 and stream_mix_small_nb.py:341-391). */
int hc_fused_bwd(const void* g_u, const void* g_x, const void* x,
                 const void* f, const float* H, const float* alpha,
                 const float* beta, void* grad_x, void* grad_f,
                 float* grad_H, float* grad_alpha, float* grad_beta,
                 int64_t T, int n, int64_t D, int stream_dtype, void* stream);

/* ===========================================================================
 * Width-read and mix + depth-write for a backbone of m blocks
 * (1 <= m <= 4, 1 <= n <= 8): the two halves of a hyper-connection layer,
 * one before and one after the wrapped module. Weights are float32, streams
 * share stream_dtype, every output is written whole.
 * ======================================================================== */

/* u[t,k,:] = sum_j R[t,k,j] x[t,j,:]      R [T,m,n], x [T,n,D] -> u [T,m,D]
 * Replaces: hyperconnections/cghc.py:410 einsum(read_in, x,
 * "b m n, b n d -> b m d"), and the same read at ghc.py:116, mhc.py:138,
 * attnhc.py:154. */
int hc_read_fwd(const float* R, const void* x, void* u, int64_t T, int n,
                int m, int64_t D, int stream_dtype, void* stream);

/* Given g_u = dL/du [T,m,D]:
 *   grad_x[t,j,:] = sum_k R[t,k,j] g_u[t,k,:]   [T,n,D] stream dtype (nullable)
 *   grad_R[t,k,j] = sum_d g_u[t,k,d] x[t,j,d]   [T,m,n] float32      (nullable)
 * Replaces the autograd backward of the read einsum (cghc.py:410). */
int hc_read_bwd(const void* g_u, const float* R, const void* x, void* grad_x,
                float* grad_R, int64_t T, int n, int m, int64_t D,
                int stream_dtype, void* stream);

/* out[t,i,:] = sum_j H_ij x_j [+ (v_i - (H v)_i) (v^T x)] + sum_k W_ik f_k
 * H [T,n,n], W [T,n,m], v [T,n] or NULL, x [T,n,D], f [T,m,D] -> out [T,n,D].
 * Replaces: cghc.py:417 einsum(write_out, out, "b n m, b m d -> b n d")
 * followed by :449 stream_mix_add (ops/stream_mix.py:57), without
 * materialising the written term Y. */
int hc_mix_write_fwd(const float* H, const void* x, const float* W,
                     const void* f, const float* v, void* out, int64_t T,
                     int n, int m, int64_t D, int stream_dtype, void* stream);

/* Given g = dL/dout [T,n,D]; with v: s = v^T x, c = v - H v, b = c^T g:
 *   grad_x_j  = sum_i H_ij g_i [+ v_j b]            [T,n,D] (nullable)
 *   grad_f_k  = sum_i W_ik g_i                      [T,m,D] (nullable)
 *   grad_H_ij = sum_d g_i (x_j [- v_j s])           [T,n,n] float32 (nullable)
 *   grad_W_ik = sum_d g_i f_k                       [T,n,m] float32 (nullable)
 *   grad_v    = rho - H^T rho + sum_d b x, rho_i = sum_d g_i s
 *                                                   [T,n]   float32 (nullable)
 * Replaces the autograd backward of the write einsum (cghc.py:417) and
 * stream_mix_small_nb.py:341-391. */
int hc_mix_write_bwd(const void* g, const float* H, const void* x,
                     const float* W, const void* f, const float* v,
                     void* grad_x, void* grad_f, float* grad_H, float* grad_W,
                     float* grad_v, int64_t T, int n, int m, int64_t D,
                     int stream_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HCOPS_H */
