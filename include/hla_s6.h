/* libhla_s6 - C ABI of the B200 (sm_100a) S6 hybrid latent-attention decode path.
 *
 * Every entry point takes plain device pointers, element strides and sizes, launches on the
 * given cudaStream_t (passed as void*), never synchronises the host and never allocates
 * device memory: outputs and the fp32 workspace are owned by the caller.  All calls are
 * safe to capture in a CUDA graph (shapes and pointers are baked in at capture; contents
 * such as ctx, block tables, q and the caches may change between replays).
 *
 * Return value: 0 on success, HLA_S6_EINVAL for a bad shape/stride/size (Python: ValueError),
 * HLA_S6_EOVERFLOW when the workspace is too small (Python: RuntimeError, the message of
 * s6_ops.S6Workspace), HLA_S6_ECUDA for a CUDA failure.  hla_s6_last_error() gives the
 * message of the calling thread's last failure.
 *
 * Data-dependent conditions are never errors: a row with no history gives o = 0 and
 * lse = -inf.  error_flag (optional, device int, may be NULL) receives a non-zero code if a
 * kernel's bounded wait ran out; the kernel then returns instead of hanging.
 *
 * Layouts (bf16 = __nv_bfloat16, unit last-dim stride everywhere):
 *   q_lat  [T, H, W]                latent query (absorbed and latent-RoPE'd)
 *   cache  [num_blocks, 1, page, 2W] latent cache, row = K (W) | V (W)
 *   block_table [T, max_blocks] int32, per token; only columns < ceil(ctx[t]/page) are read
 *               (columns at or beyond max_blocks are never read; such pages load as zeros)
 *   ctx    [T] int32 latent history rows per token
 *   lse    [H, T] fp32, natural log over already-scaled scores
 */
#ifndef HLA_S6_H
#define HLA_S6_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HLA_S6_ABI_VERSION 1
#define HLA_S6_OK 0
#define HLA_S6_EINVAL 1
#define HLA_S6_EOVERFLOW 2
#define HLA_S6_ECUDA 3

int hla_s6_version(void);
const char* hla_s6_last_error(void);

/* Fully visible attention of q_lat over the first ctx[t] paged latent rows (split-K + reduce).
 * Replaces hla/vllm_latent/s6_ops.py:117 history_attention (-> history_attention_kv :128,
 * vLLM decode_attention_fwd stage 1 + stage 2).  The workspace must hold at least
 * T * num_kv_splits * H * (W + 1) floats (s6_ops.py:109-114 S6Workspace.attn_logits).
 * out: bf16 [T, H, W] with strides (out_stride_t, out_stride_h, 1); lse: fp32 [H, T].
 * empty (optional, uint8 [T]) forces o = 0 / lse = -inf on marked rows (s6_ops.py:161). */
int hla_s6_history_attention(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                             int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row,
                             const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                             const int32_t* ctx, const uint8_t* empty, int32_t num_tokens, int32_t num_heads, int32_t width,
                             int32_t page, float scale, int32_t num_kv_splits, float* workspace,
                             int64_t workspace_floats, void* out, int64_t out_stride_t, int64_t out_stride_h,
                             float* lse, int* error_flag, void* stream);

/* Split stage only: leaves fp32 partials (o, lse per row segment) in the workspace for
 * hla_s6_history_reduce or hla_s6_decode_combine with the same (T, H, W, page, splits,
 * workspace).  Replaces the stage-1 half of s6_ops.py:156-159 (vLLM _fwd_grouped_kernel_stage1). */
int hla_s6_history_partials(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                            int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row,
                            const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                            const int32_t* ctx, int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page, float scale,
                            int32_t num_kv_splits, float* workspace, int64_t workspace_floats, int* error_flag,
                            void* stream);

/* Reduce stage: partials -> out (bf16, optional), out_f32 (fp32 [T, H, W] contiguous, optional)
 * and lse [H, T].  Replaces vLLM _decode_softmax_reducev_fwd called at s6_ops.py:158-159. */
int hla_s6_history_reduce(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page,
                          int32_t num_kv_splits, float* workspace, int64_t workspace_floats, const uint8_t* empty,
                          void* out, int64_t out_stride_t, int64_t out_stride_h, float* out_f32, float* lse,
                          void* stream);

/* Host-only: how the history kernel will partition a call (1 = stream-K over pages, 0 = one
 * CTA per row), its grid and its partial-slot capacity.  No counterpart call in the reference;
 * it exposes the split choice the reference makes in s6_ops.py:76-89 (num_kv_splits). */
int hla_s6_history_plan(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page, int32_t num_kv_splits,
                        int64_t workspace_floats, int32_t* stream_mode, int32_t* grid, int32_t* slots);

#ifdef __cplusplus
}
#endif

#endif /* HLA_S6_H */
