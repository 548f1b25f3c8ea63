/*
 * rotatek_b200 -- C ABI of the B200 (sm_100a) RotateK hot path.
 *
 * Every entry point takes plain device pointers wrapped in rtk_tensor
 * descriptors (shape + element strides), a CUDA stream as `void*`
 * (NULL = legacy default stream) and, where the kernels need scratch, a
 * caller-owned device workspace.  Nothing here allocates device memory; no
 * entry point synchronises the stream except rtk_read_status.
 *
 * Return value: RTK_OK (0) or an rtk_status code; rtk_last_error() then holds
 * a message for the calling thread.  Shape errors use the reference's
 * messages, so a host wrapper can raise them as ValueError unchanged.
 *
 * The reference (beomseokg/rotatek) is Python + Triton; each function names
 * the Python entry point it replaces.
 */
#ifndef ROTATEK_B200_H
#define ROTATEK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RTK_ABI_VERSION 1

typedef enum rtk_dtype {
  RTK_F32 = 0,
  RTK_BF16 = 1,
  RTK_F16 = 2,
  RTK_U8 = 3
} rtk_dtype;

typedef enum rtk_status {
  RTK_OK = 0,
  RTK_ERR_INVALID = 1,      /* bad shape / dtype / argument (reference: ValueError) */
  RTK_ERR_UNSUPPORTED = 2,  /* valid, but no kernel covers it                       */
  RTK_ERR_WORKSPACE = 3,    /* workspace missing or smaller than *_workspace_size() */
  RTK_ERR_CUDA = 4          /* a CUDA runtime / driver call failed                  */
} rtk_status;

/* Device-status bits a kernel may set in the workspace's status word. */
#define RTK_DEVICE_TIMEOUT 1u /* a bounded wait gave up; outputs of that call are invalid */
#define RTK_DEVICE_BAD_INPUT 2u /* rtk_spark_pack: a token's kept count differs from D_keep */

typedef struct rtk_tensor {
  void *data;          /* device pointer; NULL only where a parameter says "nullable" */
  int32_t dtype;       /* rtk_dtype */
  int32_t ndim;        /* 1..4 */
  int64_t shape[4];
  int64_t stride[4];   /* in elements */
} rtk_tensor;

/* ABI version (RTK_ABI_VERSION of the built library). */
int rtk_abi_version(void);

/* Message of the last failed call made by this thread ("" if none). */
const char *rtk_last_error(void);

/* Leave `sms` SMs (0..64, default 0) free of the tensor-core decode kernels
 * of rtk_rotatek_decode, rtk_rotatek_decode_fp8, rtk_full_channel_decode and
 * rtk_spark_decode, which otherwise launch one persistent CTA per SM.  A
 * communication kernel issued beside them -- e.g. the all_gather of one
 * layer's head-sharded outputs while the next layer decodes -- then finds SMs
 * to run on instead of waiting for the decode to finish.  Process-wide, all
 * devices; takes effect at the next call (workspaces sized with the default
 * stay large enough).  No counterpart in the reference.                       */
int rtk_decode_set_sm_reserve(int sms);

/* ------------------------------------------------------------------------
 * Decode attention
 * ------------------------------------------------------------------------ */

/* Bytes of workspace rtk_rotatek_decode needs for these shapes on `device`.
 * The first rtk_decode_workspace_counter_bytes(batch, q_heads) bytes of a
 * workspace hold counters that must read zero before a call; every call
 * leaves them zero and overwrites the bytes after them.  A workspace zeroed
 * once therefore serves any number of calls whose batch * q_heads does not
 * grow.  Calls that share a workspace must be ordered on the GPU (same
 * stream, or events): overlapping calls on one workspace race.              */
size_t rtk_rotatek_decode_workspace_size(int32_t dtype, int64_t batch, int64_t q_heads,
                                         int64_t kv_heads, int64_t head_dim,
                                         int64_t head_dim_keep, int64_t seq_full,
                                         int64_t seq_sparse, int32_t device);

/* Leading bytes of a decode workspace that must be zero before a call
 * (status word + one counter per unit; depends on batch * q_heads only).    */
size_t rtk_decode_workspace_counter_bytes(int64_t batch, int64_t q_heads);

/* Fused RotateK decode for one query token.
 * Replaces rotatek.kernels.rotatek_decode -- `paper` family
 * rotatek/kernels/fused_decode.py:303-420 (and the `gqa` twin
 * rotatek/kernels/gqa_decode.py:280-321).
 *   q_full     [B, H_q, D]              f32 | bf16 | f16
 *   R_partial  [B, H_kv, D, D_keep]     same dtype as q_full
 *   delta_mu   [B, H_kv, D]             nullable (no mean-correction bias)
 *   k_full     [B, H_kv, S_f, D]        prompt + text Keys, full width
 *   v_full     [B, H_kv, S_f, D]
 *   mask_full  [B, S_f] u8              nullable (= all ones); 0 masks a token
 *   k_sparse   [B, H_kv, S_v, D_keep]   rotated + truncated visual Keys
 *   v_sparse   [B, H_kv, S_v, D]        visual Values
 *   out        [B, H_q, D] or [B, 1, H_q, D], dtype of q_full
 * out = softmax([q.k_f * s ; (q.R.k_s + q.delta_mu) * s]) . [v_f ; v_s] / (l + 1e-6),
 * s = 1/sqrt(D), H_q = H_kv * num_kv_groups.                                 */
int rtk_rotatek_decode(const rtk_tensor *q_full, const rtk_tensor *R_partial,
                       const rtk_tensor *delta_mu, const rtk_tensor *k_full,
                       const rtk_tensor *v_full, const rtk_tensor *mask_full,
                       const rtk_tensor *k_sparse, const rtk_tensor *v_sparse,
                       int64_t num_kv_groups, const rtk_tensor *out, void *workspace,
                       size_t workspace_bytes, void *stream);

/* rtk_rotatek_decode without a workspace argument: it allocates nothing.
 * No counterpart in the reference (whose Python launcher allocates its own
 * scratch).  For callers that cannot give this library device memory -- a
 * runtime whose pool owns all of HBM and forbids outside cudaMalloc, a
 * foreign-language binding that only forwards tensor pointers, a step that
 * must not enter cudaMalloc because it can synchronise the device.
 * Its scratch is one fixed 16 MiB device array that every GPU loading the
 * library holds until the process exits; shapes needing more
 * (rtk_rotatek_decode_workspace_size) fail with RTK_ERR_WORKSPACE.  The first
 * call on a device resolves the array's address (cudaGetSymbolAddress): make
 * it before any stream capture.  All calls on a device share the array; each
 * clears its counters first, and calls that overlap on the GPU race.
 * Arguments, outputs and errors are those of rtk_rotatek_decode; the device
 * status of these calls accumulates in the array's status word, which
 * rtk_read_static_status reads.                                              */
int rtk_rotatek_decode_static(const rtk_tensor *q_full, const rtk_tensor *R_partial,
                              const rtk_tensor *delta_mu, const rtk_tensor *k_full,
                              const rtk_tensor *v_full, const rtk_tensor *mask_full,
                              const rtk_tensor *k_sparse, const rtk_tensor *v_sparse,
                              int64_t num_kv_groups, const rtk_tensor *out, void *stream);

/* rtk_rotatek_decode with the visual span stored in fp8 (e4m3, one byte per
 * element; see rtk_quantize_visual_fp8): no counterpart in the reference.
 * Visual Keys and Values are read as
 *   k~[b,h,t,c] = k_scale[b,h,c] * e4m3(k8[b,h,t,c]),   v[b,h,t,d] = v_scale[b,h,t] * e4m3(v8[b,h,d,t])
 * and the result is rtk_rotatek_decode's on those values; the prompt/text span
 * stays in q's dtype (bf16 / fp16).  Half the visual bytes of the 16-bit path.
 *   k8 [B, H_kv, S_v, D_keep] u8 (D_keep 16, 32 or 64), k_scale [B, H_kv, D_keep] f32,
 *   v8 [B, H_kv, 128, S_v] u8 (the Values transposed: token stride 1, 16-byte
 *   aligned channel rows), v_scale [B, H_kv, S_v] f32; the rest and the
 *   workspace (rtk_rotatek_decode_workspace_size) as rtk_rotatek_decode.       */
int rtk_rotatek_decode_fp8(const rtk_tensor *q_full, const rtk_tensor *R_partial,
                           const rtk_tensor *delta_mu, const rtk_tensor *k_full,
                           const rtk_tensor *v_full, const rtk_tensor *mask_full,
                           const rtk_tensor *k8, const rtk_tensor *k_scale, const rtk_tensor *v8,
                           const rtk_tensor *v_scale, int64_t num_kv_groups, const rtk_tensor *out,
                           void *workspace, size_t workspace_bytes, void *stream);

/* fp8 (e4m3) copy of a visual span for rtk_rotatek_decode_fp8: per (b, h,
 * channel) scales for the rotated Keys, per (b, h, token) scales for the
 * Values; scale = amax / 448 (1 for an all-zero group), x8 = e4m3(x / scale)
 * rounded to nearest even, saturating.
 *   k_sparse [B, H_kv, S, D_keep], v_sparse [B, H_kv, S, 128]   bf16 | f16, channel stride 1
 *   k8_out [B, H_kv, S, D_keep]: contiguous u8; v8_out [B, H_kv, 128, S] u8, the
 *   Values transposed: token stride 1, channel rows 16-byte aligned and at least
 *   S rounded up to 16 bytes long (bytes past S up to there are written as 0);
 *   k_scale_out [B, H_kv, D_keep], v_scale_out [B, H_kv, S]: contiguous f32.  */
int rtk_quantize_visual_fp8(const rtk_tensor *k_sparse, const rtk_tensor *v_sparse, const rtk_tensor *k8_out,
                            const rtk_tensor *k_scale_out, const rtk_tensor *v8_out,
                            const rtk_tensor *v_scale_out, void *stream);

/* Bytes of workspace rtk_full_channel_decode needs (same rules as above). */
size_t rtk_full_channel_decode_workspace_size(int32_t dtype, int64_t batch, int64_t q_heads,
                                              int64_t kv_heads, int64_t head_dim,
                                              int64_t seq, int32_t device);

/* Full-channel split-K flash-decode for one query token.
 * Replaces rotatek.kernels.full_channel_decode --
 * rotatek/kernels/full_channel_flash_decoding.py:162-229 (`gqa` twin
 * rotatek/kernels/gqa_decode.py:254-277).
 *   q [B, H_q, D], k / v [B, H_kv, S, D], out [B, H_q, D] or [B, 1, H_q, D]. */
int rtk_full_channel_decode(const rtk_tensor *q, const rtk_tensor *k, const rtk_tensor *v,
                            int64_t num_kv_groups, const rtk_tensor *out, void *workspace,
                            size_t workspace_bytes, void *stream);

/* SparK baseline decode without materialising its recovered Keys.
 * Replaces the adapters' SparK branch -- recovery
 * (integrations/lmms_eval/models/model_utils/llava_next/llama_visionzip.py:226-230:
 * every channel of a visual token takes its pruned-channel mean, the kept
 * channels their values), concatenation (233-234) and full_channel_decode
 * (237-242) -- with the arithmetic of that dense decode over
 * [k_full ; recovered visual Keys], [v_full ; v_sparse]; mask_full (nullable)
 * masks the prompt/text span as in rtk_rotatek_decode.
 *   k_kept [B, H_kv, S_v, D_keep]   kept channels' values in channel order
 *                                   (K_compact of rotatek/baselines/spark.py:15-58)
 *   keep_idx [B, H_kv, S_v, D_keep] their channels, uint8 ascending (rtk_spark_pack)
 *   pruned_mean [B, H_kv, S_v, 1]   per-token fill value (spark.py's pruned_mean)
 * bf16 / fp16, head_dim 128, D_keep 16, 32 or 64; 16-byte aligned,
 * channel-contiguous rows (else RTK_ERR_UNSUPPORTED).  Workspace: as for
 * rtk_rotatek_decode (rtk_rotatek_decode_workspace_size with the same shapes). */
int rtk_spark_decode(const rtk_tensor *q_full, const rtk_tensor *k_full, const rtk_tensor *v_full,
                     const rtk_tensor *mask_full, const rtk_tensor *k_kept, const rtk_tensor *keep_idx,
                     const rtk_tensor *pruned_mean, const rtk_tensor *v_sparse, int64_t num_kv_groups,
                     const rtk_tensor *out, void *workspace, size_t workspace_bytes, void *stream);

/* keep_idx_out [B, H_kv, S, D_keep] (uint8, contiguous) = each token's kept
 * channels of keep_mask [B, H_kv, S, 128] (bool as uint8, unit channel stride;
 * spark.py's keep_mask) in ascending order -- what the boolean-index
 * assignment of llama_visionzip.py:230 walks.  Run once per layer after
 * prefill.  A token whose kept count is not D_keep ORs RTK_DEVICE_BAD_INPUT
 * into *status (a device uint32; nullable). */
int rtk_spark_pack(const rtk_tensor *keep_mask, const rtk_tensor *keep_idx_out, void *status, void *stream);

/* ------------------------------------------------------------------------
 * Prefill rotation builder (head_dim 128)
 * ------------------------------------------------------------------------ */

/* cov_out[b,h] = sum_s k k^T (fp32, uncentred) and ksum_out[b,h] = sum_s k
 * over the S tokens of keys [B, H, S, 128] (f32 | bf16 | f16).  The raw sums
 * behind the covariance einsum of
 * integrations/lmms_eval/models/model_utils/kv_pruning_utils.py:112-115;
 * bf16 / fp16 keys run on the tcgen05 tensor cores.
 *   cov_out [B, H, 128, 128] f32 contiguous, ksum_out [B, H, 128] f32 contiguous. */
int rtk_key_covariance(const rtk_tensor *keys, const rtk_tensor *cov_out, const rtk_tensor *ksum_out,
                       void *stream);

/* kept_out = keys . R in the Keys' dtype: the rotation pass of
 * rtk_build_rotation on its own (kv_pruning_utils.py:152, K_vis . R on the
 * uncentred Keys), for a caller that already holds R.
 *   keys [B, H, S, 128] f32 | bf16 | f16 (any strides), R [B, H, 128, keep] and
 *   kept_out [B, H, S, keep] in the same dtype; workspace >= 256 bytes whose
 *   first word is the device-status word (see rtk_build_rotation_workspace_size). */
int rtk_rotate_keys(const rtk_tensor *keys, const rtk_tensor *R, const rtk_tensor *kept_out, void *workspace,
                    size_t workspace_bytes, void *stream);

/* Bytes of workspace rtk_eigh_topk needs for n matrices: a 256-byte head (as
 * in the build workspace); the solver keeps everything else in shared memory.
 * No zeroing required. */
size_t rtk_eigh_topk_workspace_size(int64_t n);

/* Top-k eigenvectors of symmetric matrices, descending eigenvalue, each
 * column's largest-magnitude component positive (batched 128 x 128 solver:
 * Householder tridiagonalisation, Sturm multisection, inverse iteration).
 * Replaces rotatek.rotation.power_iteration_gpu (rotatek/rotation.py:68-91),
 * which returns an unconverged basis of approximately the same subspace.
 *   cov [N, 128, 128] f32 contiguous, vecs_out [N, 128, k] f32,
 *   vals_out [N, 128] f32 contiguous (all eigenvalues, descending), nullable,
 *   workspace of rtk_eigh_topk_workspace_size(N) bytes. */
int rtk_eigh_topk(const rtk_tensor *cov, int64_t k, const rtk_tensor *vecs_out,
                  const rtk_tensor *vals_out, void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of workspace rtk_build_rotation needs: a device-status word in the
 * first 256 bytes (zero it once before first use; rtk_read_status reads and
 * clears it, a bounded wait that gave up sets RTK_DEVICE_TIMEOUT), then the
 * fp32 sums (Sum k k^T and Sum k), 66 KB per (b, h). */
size_t rtk_build_rotation_workspace_size(int64_t batch, int64_t kv_heads, int64_t head_dim);

/* The RotateK prefill build for one layer: replaces the body of
 * ChannelPruner.update_rotatek with the exact-eigh solver
 * (kv_pruning_utils.py:105-160): centred covariance of the visual Keys,
 * query weighting (when queries_recent is given), eigendecomposition, top-keep
 * rotation R, mean correction delta_mu = mu - (mu R) R^T, rotated-truncated
 * Keys kept = K_vis . R.  The keep mask (first `keep` channels) is implied.
 *   keys_vision     [B, H_kv, S_v, 128]                 f32 | bf16 | f16
 *   queries_recent  [B, H_kv * num_kv_groups, W, 128]   nullable (no weighting)
 *   kept_out        [B, H_kv, S_v, keep]                keys' dtype
 *   R_out           [B, H_kv, 128, keep]                keys' dtype
 *   delta_mu_out    [B, H_kv, 128]                      keys' dtype, nullable
 *   eigvals_out     [B, H_kv, 128] f32 contiguous       nullable (descending)   */
int rtk_build_rotation(const rtk_tensor *keys_vision, const rtk_tensor *queries_recent,
                       int64_t num_kv_groups, int64_t keep, const rtk_tensor *kept_out,
                       const rtk_tensor *R_out, const rtk_tensor *delta_mu_out,
                       const rtk_tensor *eigvals_out, void *workspace, size_t workspace_bytes,
                       void *stream);

/* The prefill Key path of the attention adapters, followed by the covariance
 * sums of its visual span.  Replaces k_proj -> view / transpose -> apply_rotary_pos_emb
 * (integrations/lmms_eval/models/model_utils/llava_next/llama_visionzip.py:144-153;
 * qwen/qwen2_5vl_visionzip.py:932-942 once the multimodal cos / sin sections are
 * merged) and the covariance pass over its visual span (kv_pruning_utils.py:112-115):
 *   keys_out[b, h, s] = k * cos + rotate_half(k) * sin,
 *   k = hidden[b, s] . w_k[h*128 : h*128 + 128]^T + bias[h*128 : ...]
 * rounded as torch rounds those bf16 / fp16 ops, for every token s; cov_out and
 * ksum_out as rtk_key_covariance over the visual tokens
 * [vis_start, vis_start + vis_len) of keys_out.  The projection, bias and
 * RoPE are one tcgen05 tensor-core kernel; the sums are then taken from the
 * visual Keys it wrote.
 *   hidden     [B, S, hidden]      bf16 | f16, hidden % 64 == 0, 16-byte aligned rows
 *   w_k        [H_kv * 128, hidden]  same dtype (nn.Linear weight)
 *   bias       [H_kv * 128]        same dtype, contiguous, nullable
 *   cos, sin   [B or 1, S, 128]    same dtype, channel stride 1
 *   keys_out   [B, H_kv, S, 128]   same dtype, channel stride 1
 *   cov_out    [B, H_kv, 128, 128] f32 contiguous; ksum_out [B, H_kv, 128] f32 contiguous
 *   workspace  rtk_key_projection_workspace_size() bytes: the device-status word
 *              (256 bytes, as in the build workspace)                            */
int rtk_key_projection(const rtk_tensor *hidden, const rtk_tensor *w_k, const rtk_tensor *bias,
                       const rtk_tensor *cos, const rtk_tensor *sin, int64_t vis_start, int64_t vis_len,
                       const rtk_tensor *keys_out, const rtk_tensor *cov_out, const rtk_tensor *ksum_out,
                       void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of workspace rtk_key_projection needs: the 256-byte status word (the
 * arguments are kept for callers that size per shape and device).            */
size_t rtk_key_projection_workspace_size(int64_t batch, int64_t kv_heads, int64_t seq, int64_t vis_start,
                                         int64_t vis_len, int32_t device);

/* Bytes of workspace rtk_build_rotation_projected needs: the build workspace
 * (rtk_build_rotation_workspace_size(batch, kv_heads, 128)).                 */
size_t rtk_build_rotation_projected_workspace_size(int64_t batch, int64_t kv_heads, int64_t seq,
                                                   int64_t vis_start, int64_t vis_len, int32_t device);

/* rtk_key_projection followed by the rest of rtk_build_rotation on the visual
 * span of keys_out: from a layer's hidden states to what the split cache stores
 * (K for every token; R, delta_mu and kept = K_vis . R for the visual span)
 * in one call; the covariance sums are taken once, by the projection step.
 * Arguments as in the two calls; kept_out is [B, H_kv, vis_len, keep];
 * workspace of rtk_build_rotation_projected_workspace_size() bytes.          */
int rtk_build_rotation_projected(const rtk_tensor *hidden, const rtk_tensor *w_k, const rtk_tensor *bias,
                                 const rtk_tensor *cos, const rtk_tensor *sin, int64_t vis_start,
                                 int64_t vis_len, const rtk_tensor *queries_recent, int64_t num_kv_groups,
                                 int64_t keep, const rtk_tensor *keys_out, const rtk_tensor *kept_out,
                                 const rtk_tensor *R_out, const rtk_tensor *delta_mu_out,
                                 const rtk_tensor *eigvals_out, void *workspace, size_t workspace_bytes,
                                 void *stream);

/* Copy the workspace's device-status word to *status (RTK_DEVICE_TIMEOUT bits)
 * and clear it.  Synchronises `stream`.                                       */
int rtk_read_status(void *workspace, void *stream, uint32_t *status);

/* rtk_read_status for rtk_rotatek_decode_static's fixed scratch on the current
 * device: the status bits its calls set since the last read, then cleared.
 * No counterpart in the reference.  Synchronises `stream`.                    */
int rtk_read_static_status(void *stream, uint32_t *status);

/* Diagnostic, no counterpart in the reference: launches one small kernel that
 * waits on an mbarrier nothing arrives on, with the bounded wait every kernel
 * here uses and a limit of limit_ns (at most 2e9) nanoseconds.  The wait gives
 * up, RTK_DEVICE_TIMEOUT is ORed into the status word at `workspace` (read it
 * with rtk_read_status), and the kernel returns: the error path of a lost TMA
 * transaction, without a copy in flight.                                      */
int rtk_selftest_wait_timeout(void *workspace, uint64_t limit_ns, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ROTATEK_B200_H */
