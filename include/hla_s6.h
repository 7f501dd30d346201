/* libhla_s6 - C ABI of the B200 (sm_100a) S6 hybrid latent-attention decode path.
 *
 * Every compute entry point takes plain device pointers, element strides and sizes, launches on
 * the given cudaStream_t (passed as void*), never synchronises the host and never allocates
 * device memory: outputs and the fp32 workspace are owned by the caller.  (The one allocating
 * call is the sequence split's set-up, hla_s6_peer_alloc.)  The compute entry points are safe to
 * capture in a CUDA graph: shapes and pointers are baked in at capture, and contents such as ctx,
 * block tables, q and the caches may change between replays.  This note does not cover
 * hla_s6_history_attention_static, whose own comment states what it needs.
 *
 * Return value: 0 on success, HLA_S6_EINVAL for a bad shape/stride/size (Python: ValueError),
 * HLA_S6_EOVERFLOW when the workspace is too small (Python: RuntimeError, the message of
 * s6_ops.S6Workspace), HLA_S6_ECUDA for a CUDA failure.  hla_s6_last_error() gives the
 * message of the calling thread's last failure.
 *
 * Data-dependent conditions are never errors: a row with no history gives o = 0 and
 * lse = -inf.  error_flag (optional, device int, may be NULL; the first code written stays)
 * receives a non-zero code when a kernel met a condition it could not honour, and the kernel
 * returns normally instead of hanging or reading outside its buffers:
 *   1, 2  a bounded wait for a shared-memory copy ran out (HLA_S6_ERR_WAIT_COPY, _WAIT_STAGE);
 *   3     a partial or a block id fell outside the workspace or the cache (HLA_S6_ERR_RANGE);
 *   4     a sequence-split part from another GPU did not arrive in time (HLA_S6_ERR_WAIT_PEER);
 *   5     a history block-table entry outside [0, num_blocks): that page reads as zeros
 *         (HLA_S6_ERR_BLOCK; the reference's torch indexing raises IndexError there).
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

#define HLA_S6_ABI_VERSION 4
#define HLA_S6_OK 0
#define HLA_S6_EINVAL 1
#define HLA_S6_EOVERFLOW 2
#define HLA_S6_ECUDA 3

#define HLA_S6_ERR_WAIT_COPY 1
#define HLA_S6_ERR_WAIT_STAGE 2
#define HLA_S6_ERR_RANGE 3
#define HLA_S6_ERR_WAIT_PEER 4
#define HLA_S6_ERR_BLOCK 5

int hla_s6_version(void);
const char* hla_s6_last_error(void);

/* Limit, in nanoseconds of device time, of every bounded wait in the kernels launched after this
 * call (mbarrier phases of the TMA rings, the sequence-split combine's wait for the other GPUs'
 * parts): when it runs out the kernel writes its error code to error_flag and returns.
 * Process-wide; 0 restores the default of 2 s.  A CUDA graph keeps the limit its launches were
 * captured with.  Returns the previous limit.  No counterpart in the reference (its Triton and
 * FA2 kernels never wait on another agent). */
uint64_t hla_s6_set_wait_limit_ns(uint64_t ns);

/* Fully visible attention of q_lat over the first ctx[t] paged latent rows (split-K + reduce).
 * Replaces hla/vllm_latent/s6_ops.py:117 history_attention (-> history_attention_kv :128,
 * vLLM decode_attention_fwd stage 1 + stage 2).  The workspace must hold at least
 * T * num_kv_splits * H * (W + 1) floats (s6_ops.py:109-114 S6Workspace.attn_logits).
 * out: bf16 [T, H, W] with strides (out_stride_t, out_stride_h, 1); lse: fp32 [H, T].
 * empty (optional, uint8 [T]) forces o = 0 / lse = -inf on marked rows (s6_ops.py:161).
 * When a step has about as many rows as the split kernel has CTAs, and the workspace holds twice
 * as many partial slots as CTAs, the split lets CTAs that finish early take the last eighth of
 * the others' pages.  Results do not depend on which CTA ran what.  The work pool's counters
 * are a pair per workspace pointer in an 8 KB device array of the library, zero between calls.
 * A pair is assigned on a workspace's first such call: make that call outside any stream
 * capture, or that one call runs without stealing. */
int hla_s6_history_attention(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                             int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row,
                             const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                             const int32_t* ctx, const uint8_t* empty, int32_t num_tokens, int32_t num_heads, int32_t width,
                             int32_t page, float scale, int32_t num_kv_splits, float* workspace,
                             int64_t workspace_floats, void* out, int64_t out_stride_t, int64_t out_stride_h,
                             float* lse, int* error_flag, void* stream);

/* hla_s6_history_attention for callers that cannot allocate device memory (a foreign-language
 * binding that is handed only input/output pointers, or a serving process whose GPU memory was
 * reserved up front): same arguments and results, minus the workspace, which is taken from a
 * fixed 8 MiB device array inside the library instead.  No counterpart in the reference.
 * Limit: T * num_kv_splits * H * (W + 1) <= 2 * 1024 * 1024 floats, else HLA_S6_EOVERFLOW.
 * The first call in each CUDA context (per device, and again after cudaDeviceReset) looks up that
 * array's device address (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the array: calls whose kernels overlap on the GPU race on it.  It allocates
 * nothing. */
int hla_s6_history_attention_static(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                                    int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row,
                                    const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                                    const int32_t* ctx, const uint8_t* empty, int32_t num_tokens, int32_t num_heads,
                                    int32_t width, int32_t page, float scale, int32_t num_kv_splits, void* out,
                                    int64_t out_stride_t, int64_t out_stride_h, float* lse, int* error_flag,
                                    void* stream);

/* Split stage only: leaves fp32 partials (o, lse per row segment) in the workspace for
 * hla_s6_history_reduce or hla_s6_decode_combine with the same (T, H, W, page, splits,
 * workspace).  Replaces the stage-1 half of s6_ops.py:156-159 (vLLM _fwd_grouped_kernel_stage1).
 * flags: HLA_S6_PARTIALS_AFTER_QUERY launches the split as a programmatic dependent of the
 * immediately preceding launch on the stream, which must be the one that writes q_lat (for example
 * hla_s6_decode_prepare) and must write nothing else this call reads: the split then streams cache
 * pages while that launch runs and reads q_lat only after it has completed. */
#define HLA_S6_PARTIALS_AFTER_QUERY 1
int hla_s6_history_partials(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                            int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row,
                            const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                            const int32_t* ctx, int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page, float scale,
                            int32_t num_kv_splits, float* workspace, int64_t workspace_floats, int* error_flag,
                            int32_t flags, void* stream);

/* Reduce stage: partials -> out (bf16, optional), out_f32 (fp32 [T, H, W] contiguous, optional)
 * and lse [H, T].  Replaces vLLM _decode_softmax_reducev_fwd called at s6_ops.py:158-159. */
int hla_s6_history_reduce(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page,
                          int32_t num_kv_splits, float* workspace, int64_t workspace_floats, const uint8_t* empty,
                          void* out, int64_t out_stride_t, int64_t out_stride_h, float* out_f32, float* lse,
                          void* stream);

/* Contiguous-layout latent history reader of the HF reference engines: per row b and head h,
 * z[b, h] = softmax_n(scale * q[b, h] . k[b, n], over keys n < num_keys with mask[b, n] != 0) . v[b, :],
 * lse[b, h] its log-sum-exp (natural log).  Rows with no visible key give z = 0, lse = -inf.
 * q bf16 [B, H, width]; k, v bf16 [B, N, width] (strides per row b and key n, unit last stride,
 * multiples of 8 elements); mask uint8 [B, N]; z bf16 [B, H, width] (strided), z32 (optional) fp32
 * [B, H, width] contiguous, lse fp32 [B, H] contiguous.  width 256, 512 or 1024; H <= 16 (MQA: one
 * K/V row shared by the heads).  The workspace follows hla_s6_history_attention's accounting
 * (B * num_kv_splits * H * (width + 1) floats).
 * Replaces the forward of hla/latent/fused_history.py:49-54 (history_attention ->
 * history_kernels.forward, history_kernels.py:11-33 and 84-89); its torch oracle is
 * fused_history.reference (fused_history.py:11-20). */
int hla_s6_history_attention_contig(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k,
                                    int64_t k_stride_b, int64_t k_stride_n, const void* v, int64_t v_stride_b,
                                    int64_t v_stride_n, const uint8_t* mask, int64_t mask_stride_b, int32_t batch,
                                    int32_t num_keys, int32_t num_heads, int32_t width, float scale,
                                    int32_t num_kv_splits, float* workspace, int64_t workspace_floats, void* z,
                                    int64_t z_stride_b, int64_t z_stride_h, float* z32, float* lse, int* error_flag,
                                    void* stream);

/* Per-head paged history (the LLA MLA-style serving path): query head h of token t attends over the
 * first ctx[t] rows of KV head h / (H / kv_heads) of cache [num_blocks, kv_heads, page, >= key_width]
 * (bf16, strides per block / head / row, unit last stride, multiples of 8 elements), scoring the
 * whole key_width row against q [T, H, key_width] and averaging its first value_width columns (the
 * row [c | rotated k_rope] read once; widths multiples of 16, value_width in {64, 128, 256, 512},
 * key_width <= 1024, page 16).
 * out bf16 [T, H, value_width] (strided), lse fp32 [H, T]; empty rows (ctx 0 or empty[t]) give
 * o = 0, lse = -inf.  Workspace: T * H * num_kv_splits * (value_width + 1) floats, the size of the
 * reference's attn_logits; within it the kernel keeps stream-K partial slots and a slot range per
 * (token, head) (num_kv_splits == 1: one slot per (token, head)).  The cache rows must be 16-byte
 * aligned; pages are read by TMA.  A block id outside the cache sets error_flag (3) and reads as zeros.
 * Replaces hla/vllm_latent/s6_ops.py:128-161 history_attention_kv(..., mla=True) (vLLM
 * decode_attention_fwd_grouped with IS_MLA), as lla_layer.attend calls it (lla_layer.py:67-74). */
int hla_s6_history_attention_heads(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                                   int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                                   int64_t cache_stride_row, int32_t kv_heads, int32_t key_width,
                                   int32_t value_width, int32_t page, const int32_t* block_table,
                                   int64_t block_table_stride, int32_t max_blocks, const int32_t* ctx,
                                   int32_t num_tokens, int32_t num_heads, float scale, int32_t num_kv_splits,
                                   float* workspace, int64_t workspace_floats, const uint8_t* empty, void* out,
                                   int64_t out_stride_t, int64_t out_stride_h, float* lse, int* error_flag,
                                   void* stream);

/* Host-only: how the history kernel will partition a call (1 = stream-K over pages, 0 = one
 * CTA per row), its grid and its partial-slot capacity.  No counterpart call in the reference;
 * it exposes the split choice the reference makes in s6_ops.py:76-89 (num_kv_splits). */
int hla_s6_history_plan(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page, int32_t num_kv_splits,
                        int64_t workspace_floats, int32_t* stream_mode, int32_t* grid, int32_t* slots);

/* Integer step metadata of a varlen batch, one launch (the integer fields of s6_layer.StepContext,
 * hla/vllm_latent/s6_layer.py:52-70, with s6_ops.token_requests :61-68 and history_lengths :71-73):
 *   token_requests[t] = #{i in 1..R : query_start_loc[i] <= t}, clamped to R - 1   (int64 [T])
 *   valid[t] = t < query_start_loc[R]; invalid[t] = !valid[t]                     (uint8 0/1 [T])
 *   history[r] = max(seq_lens[r] - (query_start_loc[r + 1] - query_start_loc[r]), 0) (int32 [R])
 *   ctx[t] = valid[t] ? history[token_requests[t]] : 0                            (int32 [T])
 *   ctx_latent[t] = window ? max(ctx[t] - window, 0) : ctx[t]                      (int32 [T])
 *   empty[t] = ctx[t] == 0; empty_latent[t] = ctx_latent[t] == 0                   (uint8 0/1 [T])
 * R = num_reqs >= 1 and query_start_loc non-decreasing (vLLM pads requests by repeating its last
 * entry).  Every output is optional (NULL skips it); seq_lens may be NULL only when history, ctx,
 * ctx_latent, empty and empty_latent all are.  Bit-exact with the reference's torch ops. */
int hla_s6_step_metadata(const int32_t* query_start_loc, int32_t num_reqs, const int32_t* seq_lens,
                         int32_t num_tokens, int32_t window, int64_t* token_requests, uint8_t* valid,
                         uint8_t* invalid, int32_t* history, int32_t* ctx, int32_t* ctx_latent, uint8_t* empty,
                         uint8_t* empty_latent, void* stream);

/* Per-token gather of a per-request block table: out[t, 0 .. max_blocks) = table[token_requests[t],
 * 0 .. max_blocks) (int32, row strides in elements); a request index outside [0, num_reqs) gives a
 * row of zeros.  Replaces s6_layer.StepContext.block_table (hla/vllm_latent/s6_layer.py:72-77,
 * table[token_requests]). */
int hla_s6_gather_block_table(const int32_t* table, int64_t table_stride, int32_t max_blocks, int32_t num_reqs,
                              const int64_t* token_requests, int32_t num_tokens, int32_t* out, int64_t out_stride,
                              void* stream);

/* Exact window attention of the roped q over keys [pos - window, pos] of a paged exact cache
 * (the current token already written; pos = seq_len - query_len + index, i.e. seq_len - 1 in
 * decode).  cache is the logical [num_blocks, H, page, 2 * head_dim] (K | V) view with strides
 * per block / head / row; block_table is per request; head_dim must be 128, window <= 127.
 * Invalid (padding) tokens give o = 0, lse = -inf.
 * Replaces hla/vllm_latent/s6_ops.py:317 window_attention_fa (FA2 varlen, window_size=[W, 0]). */
int hla_s6_window_attention(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                            int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                            int64_t cache_stride_row, int32_t page, const int32_t* block_table,
                            int64_t block_table_stride, int32_t max_blocks, const int32_t* query_start_loc,
                            int32_t num_reqs, const int32_t* seq_lens, int32_t window, float scale,
                            int32_t num_tokens, int32_t num_heads, int32_t head_dim, void* out, int64_t out_stride_t,
                            int64_t out_stride_h, float* lse, void* stream);

/* Exact window over history rows only, per token: token t reads rows [ctx[t] - window, ctx[t])
 * through row t of a per-token block table (no current token; ctx[t] = 0 gives o = 0, lse = -inf).
 * Used on prefill / mixed steps.  Replaces hla/vllm_latent/s6_ops.py:334 window_history_fa. */
int hla_s6_window_history(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                          int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                          int64_t cache_stride_row, int32_t page, const int32_t* token_block_table,
                          int64_t block_table_stride, int32_t max_blocks, const int32_t* ctx, int32_t window,
                          float scale, int32_t num_tokens, int32_t num_heads, int32_t head_dim, void* out,
                          int64_t out_stride_t, int64_t out_stride_h, float* lse, void* stream);

/* Causal attention inside each request's current chunk (cu_seqlens = query_start_loc): token i
 * attends to tokens j <= i of its request; padding tokens give o = 0, lse = -inf.  q/k/v
 * [T, H, 128] with 16-byte aligned rows; out [T, H, 128]; lse [H, T].  Replaces
 * hla/vllm_latent/s6_ops.py:234 chunk_attention (FA2 varlen causal; oracle :251-259). */
int hla_s6_chunk_attention(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                           int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                           int64_t v_stride_h, const int32_t* query_start_loc, int32_t num_reqs, int32_t num_tokens,
                           int32_t num_heads, int32_t head_dim, float scale, void* out, int64_t out_stride_t,
                           int64_t out_stride_h, float* lse, void* stream);

/* LSE merge of two partial softmaxes: +inf lse counts as empty, both empty -> 0, invalid rows
 * zeroed.  Replaces s6_ops.py:262 merge_states (vLLM merge_attn_states; oracle :275-284). */
int hla_s6_merge_states(const void* o_hist, int64_t hist_stride_t, int64_t hist_stride_h, const float* lse_hist,
                        const void* o_chunk, int64_t chunk_stride_t, int64_t chunk_stride_h, const float* lse_chunk,
                        const uint8_t* invalid, void* out, int64_t out_stride_t, int64_t out_stride_h,
                        int32_t num_tokens, int32_t num_heads, int32_t dim, void* stream);

/* LSE merge that also returns the merged lse; NaN/inf outputs of either side are sanitised.
 * Replaces s6_ops.py:353 merge_lse. */
int hla_s6_merge_lse(const void* o1, int64_t o1_stride_t, int64_t o1_stride_h, const float* lse1, const void* o2,
                     int64_t o2_stride_t, int64_t o2_stride_h, const float* lse2, void* out, int64_t out_stride_t,
                     int64_t out_stride_h, float* lse_out, int32_t num_tokens, int32_t num_heads, int32_t dim,
                     void* stream);

/* In-place neox latent RoPE of x [T, H, width] (any token/head stride) by table[positions]
 * ([max_position, width] = [cos | sin] bf16), in the torch bf16 operation order of
 * register.py:73-79.  Replaces s6_ops.py:23 latent_rope (vLLM rotary_embedding backend). */
int hla_s6_latent_rope(void* x, int64_t x_stride_t, int64_t x_stride_h, int32_t num_tokens, int32_t num_heads,
                       int32_t width, const int64_t* positions, const void* table, int64_t table_stride,
                       int64_t max_position, void* stream);

/* Latent query: out[t, h, :] = latent_rope(bf16(q_pre[t, h, :] . A[h])) with A [H, 128, width]
 * (strides a_stride_h, a_stride_k, unit last).  Replaces s6_layer.py:32 latent_query (einsum +
 * s6_ops.latent_rope). */
int hla_s6_latent_query(const void* q_pre, int64_t q_stride_t, int64_t q_stride_h, const void* A, int64_t a_stride_h,
                        int64_t a_stride_k, const int64_t* positions, const void* table, int64_t table_stride,
                        int64_t max_position, void* out, int64_t out_stride_t, int64_t out_stride_h,
                        int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t width, void* stream);

/* Exact-cache append of the current tokens: exact neox RoPE of q (in place, may be NULL) and k
 * (fp32 math, [max_position, 128] = [cos 64 | sin 64] fp32 table), then k_rope | v written at
 * slot = block_table[req, pos / page] * page + pos % page; padding tokens are skipped (slot -1).
 * slot_out (optional int64 [T]) receives the slots.  Replaces the model rotary_emb +
 * unified_kv_cache_update at hla/vllm_latent/ouro_latent.py:113-123. */
int hla_s6_exact_append(void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                        int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h, void* k_out,
                        int64_t k_out_stride_t, int64_t k_out_stride_h, const int64_t* positions,
                        const float* cos_sin, int64_t cos_sin_stride, int64_t max_position, void* cache,
                        int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                        int64_t cache_stride_row, int32_t page, const int32_t* block_table, int64_t block_table_stride,
                        int32_t max_blocks, const int32_t* query_start_loc, int32_t num_reqs, int32_t num_tokens,
                        int32_t num_heads, int32_t head_dim, int64_t* slot_out, void* stream);

/* Latent query fused with the exact-path preparation of the same (layer, loop), one launch:
 * q_lat = latent_rope(bf16(q_pre . A[h])) as hla_s6_latent_query, and, when k is not NULL,
 * q_rope = exact neox RoPE of q_pre (a separate output; q_pre is not modified) plus the
 * exact-cache append of RoPE(k) | v as hla_s6_exact_append (slot_out optional).
 * Replaces s6_layer.py:82-84 latent_query + the model rotary_emb + unified_kv_cache_update at
 * hla/vllm_latent/ouro_latent.py:112-123.  q_pre, A and latent-table rows must be 16-byte aligned.
 * flags: HLA_S6_PREPARE_EARLY_LAUNCH launches the prepare as a programmatic dependent of the
 * preceding launch on the stream: its CTAs are staged before that launch completes and wait for it
 * before they read or write memory, which hides the launch gap.  A history split launched after it
 * with HLA_S6_PARTIALS_AFTER_QUERY may then start streaming before that preceding launch has
 * completed, so the block table and ctx the split reads must not be written by it.
 * HLA_S6_PREPARE_EXACT_ONLY runs the exact part alone (k required; q_lat is not written, A is not
 * read), so that a caller can put the exact part on another stream than the latent query, e.g.
 * beside the history split with the window kernel after it; the latent query alone is the same call
 * with k = NULL. */
#define HLA_S6_PREPARE_EARLY_LAUNCH 1
#define HLA_S6_PREPARE_EXACT_ONLY 2
int hla_s6_decode_prepare(const void* q_pre, int64_t q_stride_t, int64_t q_stride_h, const void* A,
                          int64_t a_stride_h, int64_t a_stride_k, const int64_t* positions, const void* table,
                          int64_t table_stride, int64_t max_position, void* q_lat, int64_t q_lat_stride_t,
                          int64_t q_lat_stride_h, int32_t num_tokens, int32_t num_heads, int32_t head_dim,
                          int32_t width, void* q_rope, int64_t q_rope_stride_t, int64_t q_rope_stride_h,
                          const void* k, int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                          int64_t v_stride_h, const float* cos_sin, int64_t cos_sin_stride, int64_t cos_sin_rows,
                          void* cache, int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                          int64_t cache_stride_row, int32_t page, const int32_t* block_table,
                          int64_t block_table_stride, int32_t max_blocks, const int32_t* query_start_loc,
                          int32_t num_reqs, int64_t* slot_out, int32_t flags, void* stream);

/* Writer projection: reg_out = bf16(reg_in + bf16(h . weight^T)) (reg_in may be NULL), weight
 * [out_features, in_features] as nn.Linear; in_features % 128 == 0, out_features % 16 == 0.
 * Replaces register.py:45-61 write_step / write1 (cand_s[t-1](h) + previous, cand1(h)) called
 * from s6_layer.py:124 write_rows. */
int hla_s6_writer_project(const void* h, int64_t h_stride_t, const void* weight, int64_t weight_stride_n,
                          const void* reg_in, int64_t reg_in_stride_t, void* reg_out, int64_t reg_out_stride_t,
                          int32_t num_tokens, int32_t out_features, int32_t in_features, void* stream);

/* Writer projection with the row commit fused into its epilogue: the updated register
 * [T, 2w] (w = out_features / 2) is written to reg_out when that is not NULL, and committed to
 * the latent cache [num_blocks, 1, page, 2w] as hla_s6_commit_rows does (K half latent-RoPE'd
 * in the torch bf16 order, V half copied, padding tokens skipped).  Replaces
 * s6_layer.write_rows + committed_row + unified_kv_cache_update (s6_layer.py:124-147,
 * ouro_latent.py:127-129) at the commit loops. */
int hla_s6_writer_commit(const void* h, int64_t h_stride_t, const void* weight, int64_t weight_stride_n,
                         const void* reg_in, int64_t reg_in_stride_t, void* reg_out, int64_t reg_out_stride_t,
                         int32_t num_tokens, int32_t out_features, int32_t in_features, const int64_t* positions,
                         const void* table, int64_t table_stride, int64_t max_position, void* cache,
                         int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row, int32_t page,
                         const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                         const int32_t* query_start_loc, int32_t num_reqs, void* stream);

/* Committed row: row [T, 2 * width] (K | V) -> latent cache [num_blocks, 1, page, 2 * width]
 * at slot = block_table[req, pos / page] * page + pos % page with the K half latent-RoPE'd
 * (torch bf16 order) and the V half copied; padding tokens skipped.  Replaces
 * s6_layer.py:135 committed_row + unified_kv_cache_update at ouro_latent.py:127-129. */
int hla_s6_commit_rows(const void* row, int64_t row_stride_t, int32_t width, const int64_t* positions,
                       const void* table, int64_t table_stride, int64_t max_position, void* cache, int64_t num_blocks,
                       int64_t cache_stride_block, int64_t cache_stride_row, int32_t page, const int32_t* block_table,
                       int64_t block_table_stride, int32_t max_blocks, const int32_t* query_start_loc,
                       int32_t num_reqs, int32_t num_tokens, int64_t* slot_out, void* stream);

/* Fused decode tail of one (layer, loop): reduce the history partials left by
 * hla_s6_history_partials (same T, H, width, page, splits, workspace) - or, when z_in is not
 * NULL, LSE-merge num_parts reduced partials (one per GPU of a sequence-split history): part q
 * is z fp32 [T, H, width] at z_in + q * part_stride and its lse [H, T] at lse_in + q * part_stride
 * (floats; a multiple of 4) - round to bf16, up-project by
 * B [H, width, 128], run the exact window (as hla_s6_window_attention) and LSE-merge the two
 * (merge_states semantics; invalid tokens zeroed).  out bf16 [T, H, 128]; lse_out (optional
 * [H, T]) receives the merged lse.  Replaces s6_layer.py:97-115 (window_attention_fa +
 * history stage 2 + einsum B + merge_states).
 * chunk_o / chunk_lse (optional, bf16 [T, H, 128] and fp32 [H, T]): an exact part computed
 * outside (prefill / mixed steps: hla_s6_chunk_attention merged with hla_s6_window_history),
 * used instead of the decode window; the window arguments other than query_start_loc /
 * num_reqs are then ignored (s6_layer.py:101-115, non-fused branch).
 * epoch / part_seen (optional, with z_in): the parts are exchange words (HLA_S6_EXCHANGE_WORD_BYTES
 * per value; z_in, lse_in and part_stride count words, part_stride even, <= 32 parts) that other
 * GPUs store (hla_s6_history_reduce_exchange with the same slot's epoch counter).  Each word is
 * polled until it carries the tag *epoch + 1 - bounded; error_flag receives 4 and the part counts
 * as zeros on a timeout - and the combine's last CTA advances *epoch and re-zeroes the CTA counter
 * part_seen (a zeroed device int) for the slot's next exchange.
 * flags: HLA_S6_COMBINE_AFTER_PARTIALS declares that the immediately preceding launch on the
 * stream produced this combine's history input - the hla_s6_history_partials call (partials) or,
 * with z_in, the hla_s6_history_reduce_exchange call; the combine is then launched as a
 * programmatic dependent of it, and its B prefetch and exact window (whose inputs must be complete
 * before that launch) overlap the producer's tail. */
#define HLA_S6_COMBINE_AFTER_PARTIALS 1
int hla_s6_decode_combine(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t latent_page,
                          int32_t num_kv_splits, float* workspace, int64_t workspace_floats, const void* z_in,
                          const void* lse_in, int32_t num_parts, int64_t part_stride, int32_t* epoch,
                          int32_t* part_seen, const uint8_t* empty,
                          const void* B, int64_t b_stride_h,
                          int64_t b_stride_k, const void* q_rope, int64_t q_stride_t, int64_t q_stride_h,
                          const void* exact_cache, int64_t exact_num_blocks, int64_t exact_stride_block,
                          int64_t exact_stride_head, int64_t exact_stride_row, int32_t exact_page,
                          const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                          const int32_t* query_start_loc, int32_t num_reqs, const int32_t* seq_lens, int32_t window,
                          float scale, const void* chunk_o, int64_t chunk_stride_t, int64_t chunk_stride_h,
                          const float* chunk_lse, void* out, int64_t out_stride_t, int64_t out_stride_h,
                          float* lse_out, int32_t flags, int* error_flag, void* stream);

/* ---------------------------------------------------------------- sequence-split exchange
 * The reference merges a sequence-split history through NCCL (the all_gather of (z, lse) parts
 * planned for hla/vllm_latent on 8 GPUs); here the reduce stores its part straight into every
 * rank's memory over NVLink as exchange words - 8 bytes each: an fp32 value in the low 32 bits and
 * the exchange's tag in the high 32 bits - and the combine polls the words themselves, so no fence,
 * flag or collective call stands between a part's stores and its use.  The tag of a slot's k-th
 * exchange is k: every rank keeps a device int32 epoch counter per slot (zeroed, as the receive
 * slots are), which the combine advances.  A slot's next exchange must start after every rank's
 * combine of its previous one has completed (true when a step cycles through two or more slots).
 * No counterpart call in the reference. */
#define HLA_S6_EXCHANGE_WORD_BYTES 8

/* Device memory that the other processes of this node can map (CUDA IPC), zero-filled.
 * handle receives HLA_S6_PEER_HANDLE_BYTES opaque bytes to pass to hla_s6_peer_open. */
#define HLA_S6_PEER_HANDLE_BYTES 64
int hla_s6_peer_alloc(int64_t bytes, void** ptr, void* handle);
int hla_s6_peer_open(const void* handle, void** ptr);
int hla_s6_peer_close(void* ptr);
int hla_s6_peer_free(void* ptr);

/* hla_s6_history_reduce, with this GPU's reduced part (z [T, H, width] then lse [H, T], exchange
 * words tagged *epoch + 1) stored into parts[d] for every rank d < world (device pointers into each
 * rank's receive slot, this rank's own included; 16-byte aligned; T * H * width + H * T words).
 * epoch: this rank's counter for the slot, which the slot's combine (hla_s6_decode_combine with
 * the same epoch) advances.  world <= 8.
 * launch_flags: HLA_S6_REDUCE_AFTER_PARTIALS declares that the immediately preceding launch on the
 * stream is the hla_s6_history_partials call that produced the partials (the reduce is then a
 * programmatic dependent of it, and in turn lets a combine launched with
 * HLA_S6_COMBINE_AFTER_PARTIALS start its window phase while the history kernel and the reduce
 * finish: that combine's exact-window inputs must come from launches before the history call). */
#define HLA_S6_REDUCE_AFTER_PARTIALS 1
int hla_s6_history_reduce_exchange(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page,
                                   int32_t num_kv_splits, float* workspace, int64_t workspace_floats,
                                   const uint8_t* empty, uint64_t* const* parts, const int32_t* epoch,
                                   int32_t world, int32_t launch_flags, void* stream);

/* Rollout cache export: the latent rows of one finished request - positions 0 .. length-1 of every
 * layer's main cache [nb, 1, bs, main_width] and loop-1 cache [nb, 1, bs', l1_width] (bf16,
 * strides per block / row) through each kv group's physical block list (int32, device, *_blocks_len
 * entries, which must cover ceil(length / block size)) - gathered
 * into out bf16 [num_layers, length, main_width + l1_width] (main | l1 per row, contiguous), i.e.
 * the rows of the s6-rollout-cache-v1 snapshot before its device-to-host copy.  main_caches /
 * l1_caches: host arrays of num_layers (<= 64) device pointers.  A block id outside the cache sets
 * error_flag (3) and zeroes that part of the row.
 * Replaces the gather of hla/vllm_latent/cache_export.py:160-174 (RolloutCacheExporter.export). */
int hla_s6_export_rows(const void* const* main_caches, const void* const* l1_caches, int32_t num_layers,
                       int64_t main_num_blocks, int64_t main_stride_block, int64_t main_stride_row,
                       int32_t main_width, int32_t main_block_size, const int32_t* main_blocks, int64_t main_blocks_len,
                       int64_t l1_num_blocks, int64_t l1_stride_block, int64_t l1_stride_row, int32_t l1_width,
                       int32_t l1_block_size, const int32_t* l1_blocks, int64_t l1_blocks_len, int64_t length, void* out, int* error_flag,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HLA_S6_H */
