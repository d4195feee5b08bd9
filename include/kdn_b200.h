/*
 * kdn_b200 -- C ABI of the B200 (sm_100a) Kalman Delta Network scan library.
 *
 * Every entry point takes plain device pointers, int64 sizes and a CUDA stream.
 * The library never allocates or frees device memory and never synchronises:
 * the caller owns every input, output and workspace buffer (workspace sizes
 * come from the *_workspace_bytes queries) and launches are asynchronous on
 * `stream`.  Return value: KDN_OK (0) or a negative error code; the message of
 * the last error on the calling thread is kdn_last_error().
 *
 * Tensor layouts follow the reference's kdn_ops boundary: [B,T,H,D] row-major
 * contiguous for per-token vectors, [B,T,H] for per-token scalars, [H] for the
 * per-head prior.  bf16 tensors are passed as `const void*` holding
 * __nv_bfloat16.
 *
 * Each function names the reference interface it replaces
 * (path:line within ngocbh/kalman-delta-networks).
 */
#ifndef KDN_B200_H_
#define KDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kdn_stream_t; /* == cudaStream_t */

enum {
  KDN_OK = 0,
  KDN_ERR_INVALID = -1,   /* bad shape, null pointer or unsupported size */
  KDN_ERR_WORKSPACE = -2, /* workspace smaller than the query returned   */
  KDN_ERR_CUDA = -3,      /* a CUDA launch or runtime call failed        */
};

/* Version of this ABI (major * 100 + minor): 102 (101: KdnScanArgs.mode,
 * the split diagonal gain; 102: packed variable-length batches). */
int kdn_version(void);
/* Message of the last failed call on this thread ("" if none). */
const char* kdn_last_error(void);

/* ------------------------------------------------------------------------ *
 * Packed variable-length batches (the cu_seqlens convention of
 * flash-linear-attention's varlen kernels, which the reference's dense path
 * builds on; its kdn_ops entry points pass cu_seqlens=None, e.g.
 * lit_gpt/kdn_ops/iso_kdn_chunk.py:2053, diag_kdn_chunk.py:2844).  N
 * sequences lie back to back along T of a B = 1 batch; sequence i holds
 * tokens [cu_seqlens[i], cu_seqlens[i+1]) and is an independent stream: its
 * memory state and covariance start from their initial values, and its
 * 64-token chunks (and the boundary's gate prefix restarts) count from its
 * own first token.  kdn_varlen_plan builds, on the host, the int32 table
 * the varlen entry points take (copied to the device by the caller):
 *   tok[N+1] = cu_seqlens, chunk[N+1] first global chunk of each sequence,
 *   order[N] sequences by decreasing length, seq[NC] sequence of each chunk,
 * NC = sum ceil(len_i / 64).  With table == NULL it only returns NC.
 * cu_seqlens must start at 0 and increase strictly; total < 2^31.
 * ------------------------------------------------------------------------ */
int64_t kdn_varlen_table_len(int64_t num_seqs, int64_t num_chunks);
int kdn_varlen_plan(const int64_t* cu_seqlens, int64_t num_seqs, int32_t* table,
                    int64_t table_len, int64_t* num_chunks);

/* ------------------------------------------------------------------------ *
 * Isotropic gain scan.  Replaces the launches behind iso_kdn_gain
 * (lit_gpt/kdn_ops/iso_kdn_chunk.py:1966) -> _iso_kdn_gain_forward (1599) and
 * _iso_kdn_gain_backward (1797).
 *
 *   z_t = a_t p_{t-1} + omega_t,  beta_t = z_t / (r_t + z_t),
 *   p_t = r_t z_t / (r_t + posterior_scale z_t),  p_{-1} = 1/initial_precision[h]
 *
 * a, omega, r, gain, p_prev, da, domega, dr, dgain: fp32 [B,T,H].
 * initial_precision, d_initial_precision: fp32 [H].  p_prev (the covariance
 * entering each token) is written by the forward when non-null and is required
 * by the backward.  p_final (fp32 [B,H], nullable) receives p_{T-1}.
 * d_initial_precision is overwritten (not accumulated).
 * Continuation (sequence parallelism): initial_cov (fp32 [B,H], nullable)
 * replaces p_{-1} = 1/initial_precision; the backward then takes the
 * cotangent of p_{T-1} in d_final_cov (nullable = 0), writes dL/dp_{-1} to
 * d_initial_cov (nullable) and gives initial_precision no gradient.
 * Workspace: kdn_iso_gain_workspace_bytes(B, T, H) bytes of device memory
 * (the composed maps of every 16-token segment; 0 when T = 0), the same size
 * for both directions; B <= 65535.
 * ------------------------------------------------------------------------ */
size_t kdn_iso_gain_workspace_bytes(int64_t B, int64_t T, int64_t H);
int kdn_iso_gain_fwd(const float* a, const float* omega, const float* r,
                     const float* initial_precision, const float* initial_cov,
                     float* gain, float* p_prev, float* p_final, int64_t B,
                     int64_t T, int64_t H, float posterior_scale,
                     void* workspace, size_t workspace_bytes,
                     kdn_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Isotropic gate frontend.  Replaces the launches behind
 * _iso_kdn_gate_precumsum_paired (lit_gpt/kdn_ops/iso_kdn_chunk.py:1396):
 * _iso_kdn_gate_precumsum_fwd (1059) and _iso_kdn_gate_precumsum_bwd (1116).
 *
 *   g = -exp(A_log[h]) softplus(g_raw + dt_bias[h*K + k]);
 *   g_cumsum = log2(e) * (64-token-chunk-local inclusive prefix of g)  [B,T,H,K] fp32
 *   a = mean_k exp(2 g);  omega = omega_min + softplus(omega_r_raw[..., h] + omega_bias[h]);
 *   r = r_min + softplus(omega_r_raw[..., H + h] + r_bias[h])            [B,T,H] fp32
 *   initial_precision = 0.1 + softplus(initial_precision_param)          [H] fp32
 *
 * g_raw [B,T,H,K] contiguous, bf16 (g_raw_bf16 = 1) or fp32; omega_r_raw
 * [B,T,2H] bf16 or fp32 with element strides (stride_b, stride_t, 1); the five
 * parameter vectors fp32 (dt_bias [H*K]).  K is 64 or 128; B or T may be 0.
 * The backward takes the memory scan's gate cotangent dg_pre_reverse (fp32
 * [B,T,H,K], natural-log coordinates before the reverse prefix) and da,
 * domega, dr ([B,T,H]), d_initial_precision ([H]); every cotangent is
 * nullable (= zero), and every output is nullable (= not requested).  dg_raw
 * has g_raw's dtype; domega_r_raw ([B,T,2H] contiguous) has omega_r_raw's
 * dtype; the parameter gradients are fp32 and overwritten.  Workspace:
 * kdn_iso_gate_workspace_bytes(B, T, H, K) bytes (per-chunk partial sums,
 * reduced in a fixed order).
 * ------------------------------------------------------------------------ */
size_t kdn_iso_gate_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K);
int kdn_iso_gate_fwd(const void* g_raw, int g_raw_bf16, const void* omega_r_raw,
                     int omega_r_raw_bf16, int64_t omega_r_stride_b,
                     int64_t omega_r_stride_t, const float* omega_bias,
                     const float* r_bias, const float* A_log, const float* dt_bias,
                     const float* initial_precision_param, float* g_cumsum,
                     float* a, float* omega, float* r, float* initial_precision,
                     int64_t B, int64_t T, int64_t H, int64_t K, float omega_min,
                     float r_min, kdn_stream_t stream);
int kdn_iso_gate_bwd(const void* g_raw, int g_raw_bf16, const void* omega_r_raw,
                     int omega_r_raw_bf16, int64_t omega_r_stride_b,
                     int64_t omega_r_stride_t, const float* omega_bias,
                     const float* r_bias, const float* A_log, const float* dt_bias,
                     const float* initial_precision_param,
                     const float* dg_pre_reverse, const float* da,
                     const float* domega, const float* dr,
                     const float* d_initial_precision, void* dg_raw,
                     void* domega_r_raw, float* domega_bias, float* dr_bias,
                     float* dA_log, float* ddt_bias,
                     float* d_initial_precision_param, int64_t B, int64_t T,
                     int64_t H, int64_t K, void* workspace,
                     size_t workspace_bytes, kdn_stream_t stream);

/*
 * Diagonal gate / noise frontend, 32-token chunks.  Replaces
 * _diag_kdn_frontend_precumsum_paired (lit_gpt/kdn_ops/diag_kdn_chunk.py:2471):
 * forward = _frozen_frontend_diag_frontend_fwd_kernel (:1867) as launched by
 * _diag_kdn_frontend_forward (:2218); backward = _diag_kdn_frontend_backward
 * (:2265) with its alpha-presence, reduction and local VJP kernels
 * (:1908-1966, :1969).
 * retention_raw, omega_raw: bf16 [B,T,H,K]; r_raw: bf16 [B,T,H]; A_log,
 * initial_precision_param: f32 [H]; dt_bias: f32 [H,K]; all contiguous.
 * Outputs g_cumsum, alpha, omega: f32 [B,T,H,K]; r: f32 [B,T,H];
 * initial_precision: f32 [H].  Cotangents are f32 and contiguous, each may be
 * NULL (absent); gradient outputs may be NULL (not needed), but domega_raw,
 * dr_raw and d_initial_precision_param need their cotangent.  dretention_raw,
 * domega_raw, dr_raw are bf16 like their inputs.  The backward needs
 * kdn_diag_gate_workspace_bytes(B, T, H, K) bytes of workspace.
 */
size_t kdn_diag_gate_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K);
int kdn_diag_gate_fwd(const void* retention_raw, const void* omega_raw,
                      const void* r_raw, const float* A_log, const float* dt_bias,
                      const float* initial_precision_param, float* g_cumsum,
                      float* alpha, float* omega, float* r,
                      float* initial_precision, int64_t B, int64_t T, int64_t H,
                      int64_t K, kdn_stream_t stream);
int kdn_diag_gate_bwd(const void* retention_raw, const void* omega_raw,
                      const void* r_raw, const float* A_log, const float* dt_bias,
                      const float* initial_precision_param,
                      const float* d_g_cumsum, const float* d_alpha,
                      const float* d_omega, const float* d_r,
                      const float* d_initial_precision, void* dretention_raw,
                      void* domega_raw, void* dr_raw, float* dA_log,
                      float* ddt_bias, float* d_initial_precision_param,
                      int64_t B, int64_t T, int64_t H, int64_t K, void* workspace,
                      size_t workspace_bytes, kdn_stream_t stream);
int kdn_iso_gain_bwd(const float* a, const float* omega, const float* r,
                     const float* initial_precision, const float* initial_cov,
                     const float* dgain, const float* p_prev,
                     const float* d_final_cov, float* da, float* domega,
                     float* dr, float* d_initial_precision, float* d_initial_cov,
                     int64_t B, int64_t T, int64_t H, float posterior_scale,
                     void* workspace, size_t workspace_bytes,
                     kdn_stream_t stream);
/* The isotropic gain in two phases each way, for sequence parallelism (no
 * counterpart in the reference): the covariance recursion of a (b, h) stream
 * is a composition of scalar Moebius maps p -> (A p + B) / (C p + D), its
 * adjoint one of affine maps lambda -> A lambda + B, so a rank summarises
 * its segment before the covariance (or its cotangent) entering it is known:
 *   kdn_iso_gain_fwd_maps    the segment maps into the workspace and their
 *                            composition total_map (fp32 [B,H,4], scaled to
 *                            max |.| = 1);
 *   kdn_iso_gain_fwd_finish  completes kdn_iso_gain_fwd from those maps (same
 *                            workspace, untouched in between);
 *   kdn_iso_gain_bwd_maps    the adjoint maps and their composition
 *                            total_adjoint (fp32 [B,H,2]: d_initial_cov =
 *                            A d_final_cov + B);
 *   kdn_iso_gain_bwd_finish  completes kdn_iso_gain_bwd from those maps.
 * kdn_iso_gain_fwd = fwd_maps + fwd_finish, kdn_iso_gain_bwd = bwd_maps +
 * bwd_finish (without the totals); arguments as there, T > 0. */
int kdn_iso_gain_fwd_maps(const float* a, const float* omega, const float* r,
                          float* total_map, int64_t B, int64_t T, int64_t H,
                          float posterior_scale, void* workspace,
                          size_t workspace_bytes, kdn_stream_t stream);
int kdn_iso_gain_fwd_finish(const float* a, const float* omega, const float* r,
                            const float* initial_precision,
                            const float* initial_cov, float* gain, float* p_prev,
                            float* p_final, int64_t B, int64_t T, int64_t H,
                            float posterior_scale, void* workspace,
                            size_t workspace_bytes, kdn_stream_t stream);
int kdn_iso_gain_bwd_maps(const float* a, const float* omega, const float* r,
                          const float* dgain, const float* p_prev,
                          float* total_adjoint, int64_t B, int64_t T, int64_t H,
                          float posterior_scale, void* workspace,
                          size_t workspace_bytes, kdn_stream_t stream);
int kdn_iso_gain_bwd_finish(const float* a, const float* omega, const float* r,
                            const float* initial_precision,
                            const float* initial_cov, const float* dgain,
                            const float* p_prev, const float* d_final_cov, float* da,
                            float* domega, float* dr, float* d_initial_precision,
                            float* d_initial_cov, int64_t B, int64_t T, int64_t H,
                            float posterior_scale, void* workspace,
                            size_t workspace_bytes, kdn_stream_t stream);
/* The isotropic gain over a packed batch (kdn_varlen_plan): rows [1,T,H];
 * sequence i runs its own covariance stream from 1/initial_precision (or its
 * initial_cov row); initial_cov, p_final, d_final_cov, d_initial_cov are per
 * sequence, fp32 [N,H]; max_seq_len is the longest sequence (it sizes the
 * launch and kdn_iso_gain_varlen_workspace_bytes).  Same results per
 * sequence as separate calls. */
size_t kdn_iso_gain_varlen_workspace_bytes(int64_t num_seqs, int64_t max_seq_len,
                                           int64_t H);
int kdn_iso_gain_fwd_varlen(const float* a, const float* omega, const float* r,
                            const float* initial_precision,
                            const float* initial_cov, float* gain, float* p_prev,
                            float* p_final, int64_t T, int64_t H,
                            float posterior_scale, const int32_t* varlen_table,
                            int64_t num_seqs, int64_t max_seq_len, void* workspace,
                            size_t workspace_bytes, kdn_stream_t stream);
int kdn_iso_gain_bwd_varlen(const float* a, const float* omega, const float* r,
                            const float* initial_precision,
                            const float* initial_cov, const float* dgain,
                            const float* p_prev, const float* d_final_cov, float* da,
                            float* domega, float* dr, float* d_initial_precision,
                            float* d_initial_cov, int64_t T, int64_t H,
                            float posterior_scale, const int32_t* varlen_table,
                            int64_t num_seqs, int64_t max_seq_len, void* workspace,
                            size_t workspace_bytes, kdn_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Diagonal gain scan.  Replaces _diag_kdn_gain (diag_kdn_chunk.py:2737) ->
 * _diag_kdn_gain_forward (2499) / _diag_kdn_gain_backward (2569).
 *
 *   p_hat = alpha^2 p + omega,  kappa = p_hat k / (r + sum_c p_hat_c k_c^2),
 *   p <- p_hat / (1 + K k^2 / r * p_hat),  p_{-1} = 1/initial_precision[h]
 *
 * k, alpha, omega, kappa, dkappa, dk, dalpha: fp32 [B,T,H,K]; r: fp32 [B,T,H];
 * omega_raw, domega_raw: bf16 [B,T,H,K]; r_raw, dr_raw: bf16 [B,T,H];
 * initial_precision, d_initial_precision: fp32 [H].  `carry` (fp32, size from
 * kdn_diag_gain_carry_elems: the covariance entering every 64-token segment,
 * then the covariance before every token, [B,T,H,K]) is written by the
 * forward and read by the backward.  p_final (fp32 [B,H,K], nullable) receives the final covariance.
 * The backward fuses the softplus VJPs: domega_raw = dL/domega *
 * sigmoid(omega_raw), dr_raw = dL/dr * sigmoid(r_raw).  K must be 64 or 128;
 * B*H <= 65535.
 * Continuation: initial_cov (fp32 [B,H,K], nullable) replaces
 * p_{-1} = 1/initial_precision; d_final_cov / d_initial_cov (fp32 [B,H,K],
 * nullable) carry the covariance cotangent in and out, and
 * initial_precision then receives no gradient.
 * ------------------------------------------------------------------------ */
int64_t kdn_diag_gain_carry_elems(int64_t B, int64_t T, int64_t H, int64_t K);
size_t kdn_diag_gain_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t K);
int kdn_diag_gain_fwd(const float* k, const float* alpha, const float* omega,
                      const float* r, const float* initial_precision,
                      const float* initial_cov, float* kappa, float* carry,
                      float* p_final, int64_t B, int64_t T, int64_t H, int64_t K,
                      void* workspace, size_t workspace_bytes,
                      kdn_stream_t stream);
/* Allocation-free variant of kdn_diag_gain_fwd (no counterpart in the
 * reference).  For callers that must not allocate device memory at call
 * time: code running while a CUDA stream is being captured into a graph (an
 * allocation there breaks or invalidates the capture) and plugin hosts whose
 * enqueue path forbids allocation.  It takes no workspace: the per-segment
 * covariance maps live in a 16 MiB static device array of the library
 * (B*H*ceil(T/64)*K <= 1048576, larger sizes return KDN_ERR_INVALID).  It
 * calls no cudaMalloc or cudaFree.  Its first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  All calls share the array, so calls that overlap on
 * the GPU (different streams, no ordering) race; order them on one stream.
 * Outputs and carry are as for kdn_diag_gain_fwd (no initial_cov). */
int kdn_diag_gain_fwd_noalloc(const float* k, const float* alpha,
                              const float* omega, const float* r,
                              const float* initial_precision, float* kappa,
                              float* carry, float* p_final, int64_t B,
                              int64_t T, int64_t H, int64_t K,
                              kdn_stream_t stream);
/* The diagonal gain in two phases each way, for sequence parallelism (no
 * counterpart in the reference, which has no sequence parallelism).  A
 * stream's covariance recursion is a composition of per-channel Moebius maps
 * p -> (A p + B) / (C p + D), and its adjoint one of affine maps
 * lambda -> A lambda + B, so a rank can summarise its segment before the
 * covariance (or its cotangent) entering the segment is known:
 *   kdn_diag_gain_fwd_maps    writes the segment maps into the workspace and
 *                             their composition total_map (fp32 [B,H,K,4]:
 *                             A, B, C, D, scaled to max |.| = 1);
 *   kdn_diag_gain_fwd_finish  completes kdn_diag_gain_fwd from those maps
 *                             (same workspace, untouched in between);
 *   kdn_diag_gain_bwd_maps    writes the segment adjoint maps into the
 *                             workspace and their composition total_adjoint
 *                             (fp32 [B,H,K,2]: A, B with d_initial_cov =
 *                             A d_final_cov + B);
 *   kdn_diag_gain_bwd_finish  completes kdn_diag_gain_bwd from those maps.
 * kdn_diag_gain_fwd = fwd_maps + fwd_finish and kdn_diag_gain_bwd = bwd_maps
 * + bwd_finish (without the totals); arguments as there. */
int kdn_diag_gain_fwd_maps(const float* k, const float* alpha, const float* omega,
                           const float* r, float* total_map, int64_t B, int64_t T,
                           int64_t H, int64_t K, void* workspace,
                           size_t workspace_bytes, kdn_stream_t stream);
int kdn_diag_gain_fwd_finish(const float* k, const float* alpha,
                             const float* omega, const float* r,
                             const float* initial_precision,
                             const float* initial_cov, float* kappa, float* carry,
                             float* p_final, int64_t B, int64_t T, int64_t H,
                             int64_t K, void* workspace, size_t workspace_bytes,
                             kdn_stream_t stream);
int kdn_diag_gain_bwd_maps(const float* k, const float* alpha, const float* omega,
                           const float* r, const float* dkappa, const float* carry,
                           float* total_adjoint, int64_t B, int64_t T, int64_t H,
                           int64_t K, void* workspace, size_t workspace_bytes,
                           kdn_stream_t stream);
int kdn_diag_gain_bwd_finish(const float* k, const float* alpha,
                             const float* omega, const float* r,
                             const float* initial_precision,
                             const float* initial_cov, const void* omega_raw,
                             const void* r_raw, const float* dkappa,
                             const float* carry, const float* d_final_cov,
                             float* dk, float* dalpha, void* domega_raw,
                             void* dr_raw, float* d_initial_precision,
                             float* d_initial_cov, int64_t B, int64_t T, int64_t H,
                             int64_t K, void* workspace, size_t workspace_bytes,
                             kdn_stream_t stream);
int kdn_diag_gain_bwd(const float* k, const float* alpha, const float* omega,
                      const float* r, const float* initial_precision,
                      const float* initial_cov, const void* omega_raw,
                      const void* r_raw, const float* dkappa,
                      const float* carry, const float* d_final_cov, float* dk,
                      float* dalpha, void* domega_raw, void* dr_raw,
                      float* d_initial_precision, float* d_initial_cov,
                      int64_t B, int64_t T, int64_t H, int64_t K,
                      void* workspace, size_t workspace_bytes,
                      kdn_stream_t stream);
/* The diagonal gain over a packed batch (kdn_varlen_plan): B = 1, tensors
 * [1,T,H,K] / [1,T,H]; initial_cov, p_final, d_final_cov, d_initial_cov are
 * per sequence, fp32 [N,H,K]; the covariance of every sequence starts from
 * 1/initial_precision (or its initial_cov row).  Carry and workspace sizes
 * from the _varlen queries.  Same results per sequence as separate calls. */
int64_t kdn_diag_gain_varlen_carry_elems(int64_t T, int64_t H, int64_t K,
                                         int64_t num_chunks);
size_t kdn_diag_gain_varlen_workspace_bytes(int64_t T, int64_t H, int64_t K,
                                            int64_t num_chunks);
int kdn_diag_gain_fwd_varlen(const float* k, const float* alpha,
                             const float* omega, const float* r,
                             const float* initial_precision,
                             const float* initial_cov, float* kappa, float* carry,
                             float* p_final, int64_t T, int64_t H, int64_t K,
                             const int32_t* varlen_table, int64_t num_seqs,
                             int64_t num_chunks, void* workspace,
                             size_t workspace_bytes, kdn_stream_t stream);
int kdn_diag_gain_bwd_varlen(const float* k, const float* alpha,
                             const float* omega, const float* r,
                             const float* initial_precision,
                             const float* initial_cov, const void* omega_raw,
                             const void* r_raw, const float* dkappa,
                             const float* carry, const float* d_final_cov,
                             float* dk, float* dalpha, void* domega_raw,
                             void* dr_raw, float* d_initial_precision,
                             float* d_initial_cov, int64_t T, int64_t H,
                             int64_t K, const int32_t* varlen_table,
                             int64_t num_seqs, int64_t num_chunks,
                             void* workspace, size_t workspace_bytes,
                             kdn_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Diagonal q / k normalisation.  Replaces _diag_kdn_normalize
 * (lit_gpt/kdn_ops/diag_kdn_chunk.py:2162): forward kernel :194, backward
 * kernel :235 as launched by _diag_kdn_norm_backward (:2078).
 *
 *   norm = |x| over each [K] row,  d = max(norm, 1e-12),
 *   q_memory = bf16(q / d_q),  k_gain = k / d_k,  k_memory = bf16(k_gain)
 *
 * Bit-identical to the reference: round-to-nearest fp32 squares and sums in
 * its reduction order, IEEE division and square root, round-to-nearest-even
 * bf16 stores.  q_raw, k_raw: [n_rows, K] contiguous, bf16 (in_bf16 = 1) or
 * fp32; q_memory, k_memory bf16; k_gain fp32; q_norm, k_norm fp32 [n_rows]
 * (saved for the backward).  K is 64 or 128.  The backward takes the
 * cotangents of q_memory (bf16), k_gain (fp32) and k_memory (bf16), each
 * nullable (= absent), and writes dq_raw (when d_q_memory is given) and
 * dk_raw (when either key cotangent is), both in the input dtype.
 * ------------------------------------------------------------------------ */
int kdn_diag_norm_fwd(const void* q_raw, const void* k_raw, int in_bf16,
                      void* q_memory, float* k_gain, void* k_memory,
                      float* q_norm, float* k_norm, int64_t n_rows, int64_t K,
                      kdn_stream_t stream);
int kdn_diag_norm_bwd(const void* q_raw, const void* k_raw, int in_bf16,
                      const void* d_q_memory, const float* d_k_gain,
                      const void* d_k_memory, const float* q_norm,
                      const float* k_norm, void* dq_raw, void* dk_raw,
                      int64_t n_rows, int64_t K, kdn_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Gated RMS normalisation of the scan output.  Replaces the kernels behind
 * flash-linear-attention's FusedRMSNormGated / rms_norm_gated
 * (fla.modules.fused_norm_gate), the mixers' o_norm (lit_gpt/iso_kdn.py:192,
 * 305; lit_gpt/diag_kdn.py:216, 346).
 *
 *   rstd = 1 / sqrt(mean(x^2) + eps),  y = x rstd weight act(g)
 *   act = sigmoid (activation 0) or g sigmoid(g) (activation 1, "swish")
 *
 * x, y, dy, dx: [rows, D] contiguous, bf16 (x_bf16 = 1) or fp32; g, dg:
 * [rows, D], bf16 (g_bf16 = 1) or fp32; weight: fp32 [D] or NULL (no affine
 * weight); rstd: fp32 [rows] (written by the forward, read by the backward);
 * dweight: fp32 [D], overwritten, NULL when not needed (then no workspace).
 * D is 64 or 128.  Workspace: kdn_rmsnorm_gated_workspace_bytes(rows, D)
 * (per-CTA partial sums of dweight, reduced in a fixed order).
 * ------------------------------------------------------------------------ */
size_t kdn_rmsnorm_gated_workspace_bytes(int64_t rows, int64_t D);
int kdn_rmsnorm_gated_fwd(const void* x, int x_bf16, const void* g, int g_bf16,
                          const float* weight, void* y, float* rstd, int64_t rows,
                          int64_t D, float eps, int activation,
                          kdn_stream_t stream);
int kdn_rmsnorm_gated_bwd(const void* x, int x_bf16, const void* g, int g_bf16,
                          const float* weight, const void* dy, const float* rstd,
                          void* dx, void* dg, float* dweight, int64_t rows,
                          int64_t D, int activation, void* workspace,
                          size_t workspace_bytes, kdn_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Short causal depthwise convolution with SiLU in front of the scan.
 * Replaces the packed q/k/v convolution qkv_causal_conv1d
 * (lit_gpt/kdn_ops/iso_kdn_chunk.py:459, kernels behind :372 and the
 * installed causal_conv1d it calls) and the diagonal mixer's
 * _fixed_short_conv (lit_gpt/diag_kdn.py:75).
 *
 *   y[b,t,c] = silu(sum_{j<W} w[c,j] x[b, t-W+1+j, c])   (silu = 0: no activation)
 *
 * x, dx: [B,T,C] contiguous, bf16 (x_bf16 = 1) or fp32; weight, dweight:
 * [C][W] contiguous, bf16 (w_bf16 = 1) or fp32; W = 4.  The C channels are
 * `groups` (1..3) blocks of C / groups (an even count), block g written to
 * y[g] (and its cotangent read from dy[g], nullable = zero), each a
 * contiguous [B,T,C/groups] tensor of x's dtype.  dweight is overwritten.
 * Workspace: kdn_short_conv_workspace_bytes(B, T, C, W) (per-run partial
 * sums of dweight, reduced in a fixed order).
 * ------------------------------------------------------------------------ */
size_t kdn_short_conv_workspace_bytes(int64_t B, int64_t T, int64_t C, int64_t W);
int kdn_short_conv_fwd(const void* x, int x_bf16, const void* weight, int w_bf16,
                       void* const* y, int64_t groups, int64_t B, int64_t T,
                       int64_t C, int64_t W, int silu, kdn_stream_t stream);
int kdn_short_conv_bwd(const void* x, int x_bf16, const void* weight, int w_bf16,
                       const void* const* dy, int64_t groups, void* dx,
                       void* dweight, int64_t B, int64_t T, int64_t C, int64_t W,
                       int silu, void* workspace, size_t workspace_bytes,
                       kdn_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Chunked memory scan (both variants).
 *
 *   S_hat = Diag(alpha_t) S,  delta = v_t - k_t^T S_hat,
 *   S = S_hat + kappa_t delta^T,  o_t = scale q_t^T S
 *
 * variant KDN_ISO replaces _chunk_kda_precumsum_paired (iso_kdn_chunk.py:2242,
 * Function 2190): q and k are L2-normalised in the kernel (eps 1e-6),
 * kappa_t = beta_t k_hat_t, g_cumsum is 64-local, o is bf16.
 * variant KDN_DIAG replaces chunk_kalman (diag_kdn_chunk.py:3315, Function
 * 3247): q, k used as given, kappa fp32 [B,T,H,K], g_cumsum 32-local, o fp32.
 *
 * q, k, v: bf16 [B,T,H,K|V]; g_cumsum: fp32 [B,T,H,K] (base-2 chunk-local
 * inclusive prefix of ln alpha).  The backward returns dg in natural-log
 * coordinates before the reverse chunk cumsum (the reference's paired
 * cotangent, iso_kdn_chunk.py:2180-2186).
 *
 * Saved state (caller-owned, sizes from kdn_scan_saved_bytes): the forward
 * writes the chunk-start memory states and the per-chunk triangular solve and
 * query-key scores; the backward reads them.  The first 4 bytes of `saved`
 * (after kdn_scan_fwd) and of `workspace` (after kdn_scan_bwd) hold a status
 * word, zeroed by the call: bit 0 (1) is set when a bounded wait inside the
 * kernels gave up, in which case that call's results are invalid; bit 1 (2)
 * is set only when the environment variable KDN_B200_DEBUG_POLL_LIMIT = n > 0
 * is present and some wait needed more than n polls (a debug knob that lets
 * a test exercise the status check: the wait still completes and the results
 * stay valid).  Optional continuation buffers
 * (fp32 [B,H,K,V], nullable): initial_state / final_state in the forward,
 * d_final_state / d_initial_state in the backward (sequence parallelism).
 * ------------------------------------------------------------------------ */
enum { KDN_ISO = 0, KDN_DIAG = 1 };
enum { KDN_PREC_BF16 = 0, KDN_PREC_FP32 = 1 }; /* tensor-core bf16 / fp32 debug */
/* Passes a call runs (`mode`; the partial passes need KDN_PREC_BF16).  The
 * partial passes let a sequence-parallel driver summarise a segment before
 * its incoming state is known and run only the sequential pass again once it
 * is (no counterpart in the reference, which has no sequence parallelism):
 *   KDN_SCAN_FULL            both directions: every pass (the default);
 *   KDN_SCAN_FWD_RECORDS     forward: only the chunk-parallel pass, which
 *                            writes the chunk records into `saved` (no o);
 *   KDN_SCAN_FWD_SEQUENTIAL  forward: only the sequential pass (o, the saved
 *                            states, final_state) from the records an earlier
 *                            RECORDS or FULL call with the same q, k, g and
 *                            beta / kappa left in `saved`;
 *   KDN_SCAN_FWD_STATE_MAP   forward: only the segment's state map, from the
 *                            records in `saved`: final_state = the state
 *                            reached from initial_state (nullable = 0) with
 *                            the values v, final_state_map = the state reached
 *                            from the identity with zero values (the K x K
 *                            linear part, fp32 [B,H,K,K]); writes no o and no
 *                            saved states;
 *   KDN_SCAN_BWD_STATE       backward: only the reverse state sweep, writing
 *                            d_initial_state (dq ... dkappa untouched, may be
 *                            null), from the saved states of a FULL or
 *                            SEQUENTIAL forward. */
enum {
  KDN_SCAN_FULL = 0,
  KDN_SCAN_FWD_RECORDS = 1,
  KDN_SCAN_FWD_SEQUENTIAL = 2,
  KDN_SCAN_FWD_STATE_MAP = 3,
  KDN_SCAN_BWD_STATE = 4,
};

typedef struct KdnScanArgs {
  int32_t variant;   /* KDN_ISO or KDN_DIAG */
  int32_t precision; /* KDN_PREC_BF16 (product) or KDN_PREC_FP32 (debug) */
  int64_t B, T, H, K, V;
  float scale;
  /* forward inputs */
  const void* q;        /* bf16 [B,T,H,K] */
  const void* k;        /* bf16 [B,T,H,K] */
  const void* v;        /* bf16 [B,T,H,V] */
  const float* g;       /* fp32 [B,T,H,K] */
  const float* beta;    /* iso: fp32 [B,T,H] */
  const float* kappa;   /* diag: fp32 [B,T,H,K] */
  const float* initial_state; /* nullable fp32 [B,H,K,V] */
  /* forward outputs */
  void* o;              /* iso: bf16, diag: fp32 [B,T,H,V] */
  float* final_state;   /* nullable fp32 [B,H,K,V] */
  /* saved between forward and backward */
  void* saved;          /* kdn_scan_saved_bytes */
  /* backward inputs */
  const void* dO;       /* iso: bf16, diag: fp32 [B,T,H,V] */
  const float* d_final_state;   /* nullable fp32 [B,H,K,V] */
  /* backward outputs */
  void* dq;             /* bf16 [B,T,H,K] */
  void* dk;             /* bf16 [B,T,H,K] */
  void* dv;             /* bf16 [B,T,H,V] */
  float* dg;            /* fp32 [B,T,H,K] */
  float* dbeta;         /* iso: fp32 [B,T,H] */
  float* dkappa;        /* diag: fp32 [B,T,H,K] */
  float* d_initial_state;       /* nullable fp32 [B,H,K,V] */
  /* scratch */
  void* workspace;
  size_t workspace_bytes;
  /* passes to run (KDN_SCAN_*; 0 = all) and the state-map output */
  int32_t mode;
  float* final_state_map; /* KDN_SCAN_FWD_STATE_MAP: fp32 [B,H,K,K] */
  /* packed variable-length batch: the kdn_varlen_plan table on the device
   * (NULL = fixed-length batch).  Then B = 1, T = cu_seqlens[N], the bf16
   * precision and mode 0 only; initial_state, final_state, d_final_state and
   * d_initial_state are per sequence, fp32 [N,H,K,V].  Zero-initialise the
   * struct so that older callers leave this off. */
  const int32_t* varlen_table;
  int64_t num_seqs;
  int64_t num_chunks;
} KdnScanArgs;

size_t kdn_scan_saved_bytes(const KdnScanArgs* args);
size_t kdn_scan_workspace_bytes(const KdnScanArgs* args);
int kdn_scan_fwd(const KdnScanArgs* args, kdn_stream_t stream);
int kdn_scan_bwd(const KdnScanArgs* args, kdn_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* KDN_B200_H_ */
