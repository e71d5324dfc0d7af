/*
 * mhc_b200.h -- C-ABI of the B200 (sm_100a) mHC kernels.
 *
 * This is the drop-in boundary that replaces the reference's pybind11 module
 * `mhc_ascend` (ParadoxZW/mHC_Ascend, src/python/bindings.cpp:1020-1117).  Each
 * entry point below names the reference function it replaces.
 *
 * Conventions (all entry points):
 *   - Every pointer is a DEVICE pointer to contiguous row-major fp32 data
 *     (bf16 only where the name says so), on the device that is current for
 *     the calling thread.  `stream` is a cudaStream_t passed as void*.
 *   - Outputs are written, never accumulated into; the caller allocates them
 *     (the reference allocates fresh outputs with at::empty; here the Python
 *     layer allocates them with torch and passes them in).
 *   - Scalars that are parameters of the model (alpha, biases) are passed as
 *     device pointers, so a call never synchronises the host (the reference
 *     calls .item() on them: src/python/mhc/ops.py:420-422, 533-535).
 *   - Entry points that need scratch memory take (workspace, workspace_bytes)
 *     and have a *_workspace_bytes() query; they never allocate.
 *   - Return 0 (MHC_OK) on success, a negative MHC_ERR_* code otherwise;
 *     mhc_get_last_error_string() then describes the failure (per thread).
 *   - No entry point synchronises the stream or the device.
 */
#ifndef MHC_B200_H_
#define MHC_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MHC_API __attribute__((visibility("default")))
#else
#define MHC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MHC_OK 0
#define MHC_ERR_INVALID_ARG (-1)  /* bad shape / NULL pointer / bad hyper-parameter */
#define MHC_ERR_UNSUPPORTED (-2)  /* valid request this build does not implement */
#define MHC_ERR_ALIGNMENT (-3)    /* pointer not 16-byte aligned where required */
#define MHC_ERR_WORKSPACE (-4)    /* workspace NULL or smaller than *_workspace_bytes() */
#define MHC_ERR_CUDA (-5)         /* a CUDA launch reported an error */

/* Library identification and the per-thread description of the last error. */
MHC_API const char* mhc_version(void);
MHC_API const char* mhc_get_last_error_string(void);

/* ---------------------------------------------------------------------------
 * Sinkhorn-Knopp on a batch of square matrices [batch, n, n], 1 <= n <= 32.
 * Each iteration divides rows by (row sum + eps), then columns by
 * (column sum + eps) -- reference formulation ops_pytorch_backward.py:9-33.
 * ------------------------------------------------------------------------- */
/* replaces sinkhorn_knopp_fwd (bindings.cpp:155-187) */
MHC_API int mhc_sinkhorn_knopp_fwd(const float* inp, float* out, int64_t batch, int32_t n,
                           int32_t num_iters, float eps, void* stream);
/* replaces sinkhorn_knopp_bwd (bindings.cpp:189-231); exact reverse mode of
 * the forward above.  `out` (the forward result) is accepted for interface
 * parity and is not read: the forward is replayed from `inp`. */
MHC_API int mhc_sinkhorn_knopp_bwd(const float* grad_out, const float* inp, const float* out,
                           float* grad_inp, int64_t batch, int32_t n, int32_t num_iters,
                           float eps, void* stream);

/* ---------------------------------------------------------------------------
 * RMSNorm over rows of [batch, hidden]: out = inp / sqrt(mean(inp^2)+eps) * w
 * ------------------------------------------------------------------------- */
/* replaces rmsnorm_fwd (bindings.cpp:237-265); rms[batch] receives the row rms */
MHC_API int mhc_rmsnorm_fwd(const float* inp, const float* weight, float* out, float* rms,
                    int64_t batch, int64_t hidden, float eps, void* stream);
/* replaces rmsnorm_bwd (bindings.cpp:267-301).  grad_weight is a fixed-order
 * (atomic-free, deterministic) reduction over rows through the workspace. */
MHC_API size_t mhc_rmsnorm_bwd_workspace_bytes(int64_t batch, int64_t hidden);
MHC_API int mhc_rmsnorm_bwd(const float* grad_out, const float* inp, const float* weight,
                    const float* rms, float* grad_inp, float* grad_weight, int64_t batch,
                    int64_t hidden, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Stream aggregate: out[b,c] = sum_i sigmoid(H_pre_raw[b,i]) * inp[b,i,c]
 * ------------------------------------------------------------------------- */
/* replaces stream_aggregate_fwd (bindings.cpp:307-340); also writes
 * H_pre_act = sigmoid(H_pre_raw).  Output is fp32 (the reference writes bf16). */
MHC_API int mhc_stream_aggregate_fwd(const float* inp, const float* H_pre_raw, float* out,
                             float* H_pre_act, int64_t batch, int32_t n, int64_t hidden,
                             void* stream);
/* replaces stream_aggregate_bwd (bindings.cpp:342-374): grad_inp[b,i,c] =
 * H_pre_act[b,i]*grad_out[b,c]; grad_H_pre_act[b,i] = sum_c grad_out*inp. */
MHC_API int mhc_stream_aggregate_bwd(const float* grad_out, const float* inp, const float* H_pre_act,
                             float* grad_inp, float* grad_H_pre_act, int64_t batch, int32_t n,
                             int64_t hidden, void* stream);

/* ---------------------------------------------------------------------------
 * Stream distribute-mix-add:
 *   out[b,i,c] = 2*sigmoid(H_post_raw[b,i]) * y_norm[b,c] + sum_j M[b,i,j] x[b,j,c]
 * ------------------------------------------------------------------------- */
/* replaces stream_distribute_mix_add_fwd (bindings.cpp:380-412); also writes
 * H_post_act = 2*sigmoid(H_post_raw). */
MHC_API int mhc_stream_distribute_mix_add_fwd(const float* y_norm, const float* H_post_raw,
                                      const float* M, const float* x_inp, float* out,
                                      float* H_post_act, int64_t batch, int32_t n,
                                      int64_t hidden, void* stream);
/* replaces stream_distribute_mix_add_bwd (bindings.cpp:414-460): gradients
 * w.r.t. x, y_norm, M and H_post_act (the caller applies the activation
 * derivative, as ops.py:240-242 does). */
MHC_API int mhc_stream_distribute_mix_add_bwd(const float* grad_out, const float* x_inp,
                                      const float* y_norm, const float* M,
                                      const float* H_post_act, float* grad_x,
                                      float* grad_y_norm, float* grad_M,
                                      float* grad_H_post_act, int64_t batch, int32_t n,
                                      int64_t hidden, void* stream);

/* ---------------------------------------------------------------------------
 * Row RMS and the dynamic-H projection
 * ------------------------------------------------------------------------- */
/* replaces compute_rms_fwd (bindings.cpp:543-566): rms[b] = sqrt(mean(inp[b]^2)+eps) */
MHC_API int mhc_compute_rms_fwd(const float* inp, float* rms, int64_t batch, int64_t k, float eps,
                        void* stream);
/* replaces fused_rmsnorm_matmul_fwd (bindings.cpp:480-528): out[b,o] =
 * sum_k inp[b,k]*weight[o,k], computed in fp32 (the reference casts to bf16). */
MHC_API int mhc_fused_rmsnorm_matmul_fwd(const float* inp, const float* weight, float* out,
                                 int64_t batch, int64_t k, int32_t out_dim, void* stream);
/* replaces fused_rmsnorm_matmul_bwd (bindings.cpp:530-541): grad_inp =
 * grad_out @ weight, grad_weight = grad_out^T @ inp (fixed-order reduction). */
MHC_API size_t mhc_fused_rmsnorm_matmul_bwd_workspace_bytes(int64_t batch, int64_t k, int32_t out_dim);
MHC_API int mhc_fused_rmsnorm_matmul_bwd(const float* grad_out, const float* inp, const float* weight,
                                 float* grad_inp, float* grad_weight, int64_t batch, int64_t k,
                                 int32_t out_dim, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* ---------------------------------------------------------------------------
 * MHCResidualWrapper in one piece (replaces layer.py:287-316 around the fused
 * layer, bindings.cpp:600-952): for n = 4, fp32, hidden % 32 == 0 and 16-byte
 * aligned tensors, the streams are built inside the layer kernels from
 * residual / branch ([tokens, hidden] each; stream i = scales[i] * residual,
 * stream 1 = branch, exactly as mhc_wrapper_pack_fwd computes them) and the
 * forward writes the stream mean out_mean [tokens, hidden] -- the packed input
 * and the layer output never reach memory.  Workspaces and token_state as for
 * mhc_layer_fwd_dynamic / mhc_layer_bwd_dynamic with batch = tokens.  The
 * backward takes the mean's gradient and writes the residual and branch
 * gradients plus the parameter gradients (written, not accumulated).  Other
 * shapes return MHC_ERR_UNSUPPORTED (use the pack / layer / mean entry points).
 * ------------------------------------------------------------------------- */
MHC_API int mhc_wrapper_fwd_dynamic(const float* residual, const float* branch, const float* scales,
                                    const float* rmsnorm_weight, const float* phi_pre,
                                    const float* phi_post, const float* phi_res,
                                    const float* alpha_pre, const float* alpha_post,
                                    const float* alpha_res, const float* b_pre,
                                    const float* b_post, const float* b_res, float* out_mean,
                                    float* token_state, int64_t tokens, int32_t n, int64_t hidden,
                                    int32_t sinkhorn_iters, float sinkhorn_eps, float rmsnorm_eps,
                                    void* workspace, size_t workspace_bytes, void* stream);
/* The wrapper forward fused with the next branch's input RMSNorm (a pre-norm
 * block normalises the returned hidden state before its attention / MLP; the
 * reference composes MHCResidualWrapper.forward (layer.py:287-316) with the
 * branch's rmsnorm (ops.py:87-136) as two passes).  Writes out_mean as
 * mhc_wrapper_fwd_dynamic does, and out_normed[t, c] = out_mean[t, c] /
 * out_norm_rms[t] * norm_weight[c], out_norm_rms[t] = sqrt(mean_c out_mean^2
 * + norm_eps), from the same pass.  The backward of the norm is
 * mhc_rmsnorm_bwd on (grad_normed, out_mean, norm_weight, out_norm_rms); its
 * input gradient adds to grad_mean of mhc_wrapper_bwd_dynamic.  Same
 * requirements and workspace as mhc_wrapper_fwd_dynamic; norm_weight and
 * out_normed 16-byte aligned. */
MHC_API int mhc_wrapper_fwd_dynamic_prenorm(
    const float* residual, const float* branch, const float* scales, const float* rmsnorm_weight,
    const float* phi_pre, const float* phi_post, const float* phi_res, const float* alpha_pre,
    const float* alpha_post, const float* alpha_res, const float* b_pre, const float* b_post,
    const float* b_res, const float* norm_weight, float norm_eps, float* out_mean,
    float* out_normed, float* out_norm_rms, float* token_state, int64_t tokens, int32_t n,
    int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps, float rmsnorm_eps,
    void* workspace, size_t workspace_bytes, void* stream);
MHC_API int mhc_wrapper_bwd_dynamic(const float* grad_mean, const float* residual,
                                    const float* branch, const float* scales,
                                    const float* rmsnorm_weight, const float* phi_pre,
                                    const float* phi_post, const float* phi_res,
                                    const float* alpha_pre, const float* alpha_post,
                                    const float* alpha_res, const float* b_pre,
                                    const float* b_post, const float* b_res,
                                    const float* token_state, float* grad_residual,
                                    float* grad_branch, float* grad_rmsnorm_weight,
                                    float* grad_phi_pre, float* grad_phi_post, float* grad_phi_res,
                                    float* grad_alpha_pre, float* grad_alpha_post,
                                    float* grad_alpha_res, float* grad_b_pre, float* grad_b_post,
                                    float* grad_b_res, int64_t tokens, int32_t n, int64_t hidden,
                                    int32_t sinkhorn_iters, float sinkhorn_eps, float rmsnorm_eps,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * MHCResidualWrapper stream packing and stream mean (replace the framework ops
 * of layer.py:287-316; the reference has no native counterpart).  Tokens are
 * the flattened leading dims, x is [tokens, n, hidden] fp32, n <= 64.
 * scales: host array of n floats; stream i (i != 1) is scales[i] * residual
 * (scales[0] is taken as 1; "decay" mode passes 0.1^(i-1), "zero" mode 0, and
 * a zero scale writes 0).  Stream 1 is the branch output.
 * ------------------------------------------------------------------------- */
MHC_API int mhc_wrapper_pack_fwd(const float* residual, const float* branch, float* out,
                                 const float* scales, int64_t tokens, int32_t n, int64_t hidden,
                                 void* stream);
/* bf16 residual / branch_output (tokens x hidden bf16, 8-byte aligned for the
 * vector path), fp32 streams out: the reference packs in residual.dtype
 * (layer.py:299-308), so streams i >= 2 are scales[i] * residual rounded to
 * bf16 before the layer widens them (layer.py:101). */
MHC_API int mhc_wrapper_pack_fwd_bf16(const void* residual, const void* branch, float* out,
                                      const float* scales, int64_t tokens, int32_t n,
                                      int64_t hidden, void* stream);
/* grad_residual = sum_{i != 1} scales[i] * grad[:, i]; grad_branch = grad[:, 1] (may be NULL) */
MHC_API int mhc_wrapper_pack_bwd(const float* grad_out, float* grad_residual, float* grad_branch,
                                 const float* scales, int64_t tokens, int32_t n, int64_t hidden,
                                 void* stream);
/* out[t, c] = mean_i inp[t, i, c]  (MHCResidualWrapper's output.mean(dim=1)) */
MHC_API int mhc_stream_mean_fwd(const float* inp, float* out, int64_t tokens, int32_t n,
                                int64_t hidden, void* stream);
/* grad_inp[t, i, c] = grad_out[t, c] / n */
MHC_API int mhc_stream_mean_bwd(const float* grad_out, float* grad_inp, int64_t tokens, int32_t n,
                                int64_t hidden, void* stream);

/* ---------------------------------------------------------------------------
 * Fused mHC layer, dynamic H.
 *
 * Per-token record saved by the forward for the backward ("token_state",
 * [batch, mhc_token_state_stride(n)] fp32):
 *   [0] rms_h  (rms of the flattened n*C token vector)
 *   [1] rms    (rms of the aggregated stream, RMSNorm denominator)
 *   [2, 2+n)          H_pre_act  = sigmoid(H_pre_tilde)
 *   [2+n, 2+2n)       H_post_act = 2*sigmoid(H_post_tilde)
 *   [2+2n, 2+2n+n*n)  M          = Sinkhorn(exp(H_res_tilde))
 *   [2+2n+n*n, ...+n*n+2n)  raw projections p = x_flat @ phi^T (pre|post|res)
 *   then, from the next even index, n(n+1)/2 doubles: the upper triangle of
 *   the token's Gram matrix x x^T (row-major), accumulated in fp64 from exact
 *   products; the record (and therefore the buffer) must be 8-byte aligned.
 *   Stride at n = 4: 72 floats.
 * ------------------------------------------------------------------------- */
MHC_API int32_t mhc_token_state_stride(int32_t n);

/* replaces mhc_layer_fwd_dynamic (bindings.cpp:880-952).  alpha_* point to
 * one device float each; b_res is [n,n].  token_state may be NULL for
 * inference (nothing saved).  1 <= n <= 32; which kernels run depends on n and
 * batch (n >= 8, or n = 6, 7 from 1024 tokens: the wide-rate set), so the
 * workspace size must come from the same (batch, n, hidden). */
MHC_API size_t mhc_layer_fwd_dynamic_workspace_bytes(int64_t batch, int32_t n, int64_t hidden);
MHC_API int mhc_layer_fwd_dynamic(const float* x, const float* rmsnorm_weight, const float* phi_pre,
                          const float* phi_post, const float* phi_res, const float* alpha_pre,
                          const float* alpha_post, const float* alpha_res, const float* b_pre,
                          const float* b_post, const float* b_res, float* out,
                          float* token_state, int64_t batch, int32_t n, int64_t hidden,
                          int32_t sinkhorn_iters, float sinkhorn_eps, float rmsnorm_eps,
                          void* workspace, size_t workspace_bytes, void* stream);

/* bf16 streams, an extension of mhc_layer_fwd_dynamic (the reference
 * keeps bf16 intermediates, bindings.cpp:906): x and out are bf16, the
 * parameters, token_state and all arithmetic fp32.  Needs n <= 4, hidden a
 * multiple of 64 and 16-byte aligned x / out / rmsnorm_weight
 * (MHC_ERR_UNSUPPORTED / MHC_ERR_ALIGNMENT otherwise).  Workspace as for
 * mhc_layer_fwd_dynamic. */
MHC_API int mhc_layer_fwd_dynamic_bf16(const void* x, const float* rmsnorm_weight,
                          const float* phi_pre, const float* phi_post, const float* phi_res,
                          const float* alpha_pre, const float* alpha_post,
                          const float* alpha_res, const float* b_pre, const float* b_post,
                          const float* b_res, void* out, float* token_state, int64_t batch,
                          int32_t n, int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps,
                          float rmsnorm_eps, void* workspace, size_t workspace_bytes,
                          void* stream);

/* No counterpart in the reference.  Same as mhc_layer_fwd_dynamic, for
 * callers that cannot provide a workspace (no device allocator of their own,
 * device memory fixed at start-up, or a path that must not call cudaMalloc /
 * cudaFree because they can synchronise the device): the scratch comes from
 * a 16 MiB array in the library's device image, which every GPU that loads
 * the library holds until the process exits.  Requests needing more than
 * 16 MiB return MHC_ERR_UNSUPPORTED; the need depends on the shape, on
 * whether token_state is given (without it the record is scratch too) and on
 * the SM count -- on a 148-SM B200 at n=4, C=4096 about 20k tokens fit with a
 * token_state and about 16k without.  The first call on a
 * device looks up the array's device address (make it before any stream
 * capture).  All calls on a device share the array: calls whose kernels may
 * overlap on the GPU race and must be serialised by the caller. */
MHC_API int mhc_layer_fwd_dynamic_noalloc(const float* x, const float* rmsnorm_weight,
                                          const float* phi_pre, const float* phi_post,
                                          const float* phi_res, const float* alpha_pre,
                                          const float* alpha_post, const float* alpha_res,
                                          const float* b_pre, const float* b_post,
                                          const float* b_res, float* out, float* token_state,
                                          int64_t batch, int32_t n, int64_t hidden,
                                          int32_t sinkhorn_iters, float sinkhorn_eps,
                                          float rmsnorm_eps, void* stream);

/* replaces mhc_layer_bwd_dynamic (bindings.cpp:600-874).  All parameter
 * gradients are written (not accumulated); they are fixed-order reductions
 * over the batch, so results are bitwise reproducible run to run. */
MHC_API size_t mhc_layer_bwd_dynamic_workspace_bytes(int64_t batch, int32_t n, int64_t hidden);
MHC_API int mhc_layer_bwd_dynamic(const float* grad_out, const float* x, const float* rmsnorm_weight,
                          const float* phi_pre, const float* phi_post, const float* phi_res,
                          const float* alpha_pre, const float* alpha_post,
                          const float* alpha_res, const float* b_pre, const float* b_post,
                          const float* b_res, const float* token_state, float* grad_x,
                          float* grad_rmsnorm_weight, float* grad_phi_pre,
                          float* grad_phi_post, float* grad_phi_res, float* grad_alpha_pre,
                          float* grad_alpha_post, float* grad_alpha_res, float* grad_b_pre,
                          float* grad_b_post, float* grad_b_res, int64_t batch, int32_t n,
                          int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps,
                          float rmsnorm_eps, void* workspace, size_t workspace_bytes,
                          void* stream);

/* bf16 streams for the backward: grad_out, x and grad_x are bf16, every
 * parameter gradient fp32 (arithmetic fp32, moments fp64 as in
 * mhc_layer_bwd_dynamic).  Needs n == 4, hidden a multiple of 32 and 16-byte
 * aligned tensors.  Workspace as for mhc_layer_bwd_dynamic. */
MHC_API int mhc_layer_bwd_dynamic_bf16(const void* grad_out, const void* x,
                          const float* rmsnorm_weight, const float* phi_pre,
                          const float* phi_post, const float* phi_res,
                          const float* alpha_pre, const float* alpha_post,
                          const float* alpha_res, const float* b_pre, const float* b_post,
                          const float* b_res, const float* token_state, void* grad_x,
                          float* grad_rmsnorm_weight, float* grad_phi_pre,
                          float* grad_phi_post, float* grad_phi_res, float* grad_alpha_pre,
                          float* grad_alpha_post, float* grad_alpha_res, float* grad_b_pre,
                          float* grad_b_post, float* grad_b_res, int64_t batch, int32_t n,
                          int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps,
                          float rmsnorm_eps, void* workspace, size_t workspace_bytes,
                          void* stream);

/* ---------------------------------------------------------------------------
 * Fused mHC layer, static H (shared logits H_pre[n], H_post[n], H_res[n,n]).
 * The reference composes this from four operators (layer.py:142-170); these
 * entry points run the same math as one forward kernel and a fused backward.
 * The forward saves rms[batch] (RMSNorm denominators) when rms != NULL.
 * x/out are fp32 (..._f32) or bf16 with fp32 arithmetic (..._bf16).
 * ------------------------------------------------------------------------- */
MHC_API size_t mhc_layer_static_workspace_bytes(int64_t batch, int32_t n, int64_t hidden);
MHC_API int mhc_layer_fwd_static_f32(const float* x, const float* rmsnorm_weight, const float* H_pre,
                             const float* H_post, const float* H_res, float* out, float* rms,
                             int64_t batch, int32_t n, int64_t hidden, int32_t sinkhorn_iters,
                             float sinkhorn_eps, float rmsnorm_eps, void* workspace,
                             size_t workspace_bytes, void* stream);
MHC_API int mhc_layer_fwd_static_bf16(const void* x, const float* rmsnorm_weight, const float* H_pre,
                              const float* H_post, const float* H_res, void* out, float* rms,
                              int64_t batch, int32_t n, int64_t hidden, int32_t sinkhorn_iters,
                              float sinkhorn_eps, float rmsnorm_eps, void* workspace,
                              size_t workspace_bytes, void* stream);
MHC_API int mhc_layer_bwd_static(const float* grad_out, const float* x, const float* rmsnorm_weight,
                         const float* H_pre, const float* H_post, const float* H_res,
                         const float* rms, float* grad_x, float* grad_rmsnorm_weight,
                         float* grad_H_pre, float* grad_H_post, float* grad_H_res,
                         int64_t batch, int32_t n, int64_t hidden, int32_t sinkhorn_iters,
                         float sinkhorn_eps, float rmsnorm_eps, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Device error word.  No counterpart in the reference.  Kernels that wait on
 * asynchronous copies (TMA + mbarrier) bound every wait; a wait that runs out
 * sets this word to nonzero and the kernel abandons its work (its outputs are
 * then incomplete) instead of hanging the GPU.  Reads the word (synchronous
 * copy from the device) and optionally resets it to zero.
 * ------------------------------------------------------------------------- */
MHC_API int mhc_device_error_word(int32_t* value, int32_t reset);

/* ---------------------------------------------------------------------------
 * Kernel timing (tracing).  No counterpart in the reference, which times
 * whole calls from Python (benchmark.py:156-269).  While enabled, every kernel
 * this library launches is bracketed by two CUDA events on its own stream;
 * mhc_profile_report() waits for them and writes one line per kernel name:
 * "<name> <launches> <total_ms>\n" (NUL-terminated, truncated to cap), then
 * clears the record.  Returns the number of bytes written, or < 0 on error.
 * Process-wide; meant for benchmarking, not for concurrent production use.
 * ------------------------------------------------------------------------- */
MHC_API int mhc_profile_enable(int enable);
MHC_API int mhc_profile_report(char* buf, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* MHC_B200_H_ */
