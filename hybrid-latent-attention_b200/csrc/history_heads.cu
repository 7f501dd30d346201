// Per-head paged history reader: the LLA MLA-style serving path.
//
// Reference behaviour: hla/vllm_latent/s6_ops.py:128-161 history_attention_kv(..., mla=True), called
// by lla_layer.attend (lla_layer.py:67-74) with k = cache[..., :r + d_rope] and v = cache[..., :r] of a
// per-head latent cache [num_blocks, kvH, block, r + d_rope]: each query head h attends over the
// first ctx[t] rows of KV head h / (H / kvH); the K row is the whole [c | rotated k_rope] row, V its
// first r columns, so every row is read once (vLLM's grouped decode kernel with IS_MLA).  Its torch
// oracle is _history_reference (s6_ops.py:204-222).  Empty rows give o = 0, lse = -inf.
//
// B200 design.  With a KV head per query head (LLA: kvH = H = 16) each (token, head) pair is a GEMV
// at ~1 flop per byte, an HBM stream that CUDA cores sustain; the heads-as-M tensor-core tiling of the
// MQA reader does not apply.  One CTA per (token, head, split): a cp.async ring stages the head's
// pages (16 rows x Lk) in shared memory, rows past ctx zero-filled; warps score 4 keys each (lanes
// over columns, warp-sum), the CTA keeps the online softmax, and every thread accumulates its Lv
// columns of P.V from the same tile.  The normalised partial and its lse go to the workspace
// [T, H, splits, Lv + 1] (the reference's attn_logits layout); a second kernel merges the splits.
#include "../../include/hla_s6.h"
#include "common.cuh"
#include "hla_s6_internal.h"

namespace hla {

constexpr int kHdThreads = 128, kHdStages = 4, kHdPage = 16, kHdMaxCols = 4;  // Lv <= 512

struct HeadsParams {
  const __nv_bfloat16* q;  // [T, H, Lk]
  int64_t q_st, q_sh;
  const __nv_bfloat16* cache;  // [nb, kvH, page, >= Lk]; V = first Lv columns of each row
  int64_t c_sb, c_sh, c_sr, nb;
  const int32_t* bt;
  int64_t bt_st;
  int max_blocks;
  const int32_t* ctx;
  int T, H, kvH, Lk, Lv, splits;
  float scale_log2;
  float* ws;  // [T, H, splits, Lv + 1]
  int* err;
};

__global__ void __launch_bounds__(kHdThreads) history_heads_split_kernel(const HeadsParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x % p.splits;
  const int row = blockIdx.x / p.splits;  // t * H + h
  const int t = row / p.H, h = row % p.H;
  const int kvh = h / (p.H / p.kvH);
  const int Lk = p.Lk, Lv = p.Lv, lk8 = Lk / 8;
  const int tile_bytes = kHdPage * Lk * 2;
  uint8_t* tiles = smem_raw;
  float* qs = reinterpret_cast<float*>(smem_raw + kHdStages * tile_bytes);  // [Lk]
  float* sc = qs + Lk;                                                      // [16] scores (log2 domain)
  float* out = p.ws + (static_cast<int64_t>(row) * p.splits + split) * (Lv + 1);

  const int n = max(p.ctx[t], 0);
  const int pages = (n + kHdPage - 1) / kHdPage;
  const int per = (pages + p.splits - 1) / p.splits;
  const int pg0 = split * per, pg1 = min(pages, pg0 + per);
  if (pg0 >= pg1) {  // nothing to read in this split
    for (int c = tid; c < Lv; c += kHdThreads) out[c] = 0.f;
    if (tid == 0) out[Lv] = -INFINITY;
    return;
  }
  const __nv_bfloat16* qr = p.q + static_cast<int64_t>(t) * p.q_st + static_cast<int64_t>(h) * p.q_sh;
  for (int c = tid; c < Lk; c += kHdThreads) qs[c] = __bfloat162float(qr[c]) * p.scale_log2;

  auto load_page = [&](int lp, int stage) {
    int blk = lp < p.max_blocks ? p.bt[static_cast<int64_t>(t) * p.bt_st + lp] : -1;
    if (blk < 0 || blk >= p.nb) {
      if (tid == 0) record_error(p.err, kErrSlots);
      blk = -1;
    }
    const int valid = min(kHdPage, n - lp * kHdPage);
    uint8_t* dst = tiles + stage * tile_bytes;
    const __nv_bfloat16* base = p.cache + static_cast<int64_t>(blk < 0 ? 0 : blk) * p.c_sb +
                                static_cast<int64_t>(kvh) * p.c_sh;
    for (int i = tid; i < kHdPage * lk8; i += kHdThreads) {
      const int r = i / lk8, ch = i % lk8;
      const bool live = blk >= 0 && r < valid;  // rows past ctx (and unreadable blocks) read as zeros
      cp_async16(dst + (r * Lk + ch * 8) * 2, base + static_cast<int64_t>(live ? r : 0) * p.c_sr + ch * 8,
                 live ? 16 : 0);
    }
  };

  // prologue: STAGES - 1 pages in flight
#pragma unroll
  for (int s = 0; s < kHdStages - 1; ++s) {
    if (pg0 + s < pg1) load_page(pg0 + s, s);
    cp_async_commit();
  }
  __syncthreads();  // q staged

  float m = -INFINITY, l = 0.f;
  float o[kHdMaxCols];
#pragma unroll
  for (int i = 0; i < kHdMaxCols; ++i) o[i] = 0.f;

  for (int lp = pg0, it = 0; lp < pg1; ++lp, ++it) {
    const int nxt = lp + kHdStages - 1;
    if (nxt < pg1) load_page(nxt, (it + kHdStages - 1) % kHdStages);
    cp_async_commit();
    cp_async_wait<kHdStages - 1>();
    __syncthreads();
    const __nv_bfloat16* tile = reinterpret_cast<const __nv_bfloat16*>(tiles + (it % kHdStages) * tile_bytes);
    const int valid = min(kHdPage, n - lp * kHdPage);
    // scores: warp w owns keys 4w .. 4w + 3
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int key = warp * 4 + kk;
      const __nv_bfloat162* kr = reinterpret_cast<const __nv_bfloat162*>(tile + key * Lk);
      float acc = 0.f;
      for (int c = lane; c < Lk / 2; c += 32) {
        const float2 kv = __bfloat1622float2(kr[c]);
        acc = fmaf(qs[2 * c], kv.x, fmaf(qs[2 * c + 1], kv.y, acc));
      }
      acc = warp_sum(acc);
      if (lane == 0) sc[key] = key < valid ? acc : -INFINITY;
    }
    __syncthreads();
    float tmax = -INFINITY;
#pragma unroll
    for (int k = 0; k < kHdPage; ++k) tmax = fmaxf(tmax, sc[k]);
    const float mn = fmaxf(m, tmax);  // finite: every visited page has a key below ctx
    const float alpha = exp2f(m - mn);
    float pk[kHdPage];
    float ps = 0.f;
#pragma unroll
    for (int k = 0; k < kHdPage; ++k) {
      pk[k] = exp2f(sc[k] - mn);
      ps += pk[k];
    }
    l = l * alpha + ps;
    m = mn;
#pragma unroll
    for (int i = 0; i < kHdMaxCols; ++i) {
      const int c = tid + i * kHdThreads;
      if (c < Lv) {
        float acc = o[i] * alpha;
#pragma unroll
        for (int k = 0; k < kHdPage; ++k) acc = fmaf(pk[k], __bfloat162float(tile[k * Lk + c]), acc);
        o[i] = acc;
      }
    }
    __syncthreads();  // the tile and the scores are consumed
  }
  cp_async_wait<0>();
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int i = 0; i < kHdMaxCols; ++i) {
    const int c = tid + i * kHdThreads;
    if (c < Lv) out[c] = o[i] * inv;
  }
  if (tid == 0) out[Lv] = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
}

// Merge of a (token, head)'s splits -> o (bf16, [T, H, Lv] strided) and lse [H, T].
__global__ void __launch_bounds__(kHdThreads) history_heads_reduce_kernel(const float* __restrict__ ws, int H,
                                                                          int T, int splits, int Lv,
                                                                          const uint8_t* __restrict__ empty,
                                                                          __nv_bfloat16* __restrict__ out,
                                                                          int64_t o_st, int64_t o_sh,
                                                                          float* __restrict__ lse) {
  const int row = blockIdx.x, t = row / H, h = row % H, tid = threadIdx.x;
  const float* base = ws + static_cast<int64_t>(row) * splits * (Lv + 1);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, base[static_cast<int64_t>(s) * (Lv + 1) + Lv]);
  const bool is_empty = (empty && empty[t]) || mx == -INFINITY;
  float wsum = 0.f;
  float acc[kHdMaxCols] = {0.f, 0.f, 0.f, 0.f};
  if (!is_empty) {
    for (int s = 0; s < splits; ++s) {
      const float* part = base + static_cast<int64_t>(s) * (Lv + 1);
      const float w = expf(part[Lv] - mx);  // 0 for an empty split
      wsum += w;
#pragma unroll
      for (int i = 0; i < kHdMaxCols; ++i) {
        const int c = tid + i * kHdThreads;
        if (c < Lv && w > 0.f) acc[i] = fmaf(w, part[c], acc[i]);
      }
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  __nv_bfloat16* dst = out + static_cast<int64_t>(t) * o_st + static_cast<int64_t>(h) * o_sh;
#pragma unroll
  for (int i = 0; i < kHdMaxCols; ++i) {
    const int c = tid + i * kHdThreads;
    if (c < Lv) dst[c] = __float2bfloat16_rn(is_empty ? 0.f : acc[i] * inv);
  }
  if (tid == 0) lse[static_cast<int64_t>(h) * T + t] = is_empty ? -INFINITY : mx + logf(wsum);
}

}  // namespace hla

using namespace hla;

extern "C" int hla_s6_history_attention_heads(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                                              const void* cache, int64_t num_blocks, int64_t cache_stride_block,
                                              int64_t cache_stride_head, int64_t cache_stride_row, int32_t kv_heads,
                                              int32_t key_width, int32_t value_width, int32_t page,
                                              const int32_t* block_table, int64_t block_table_stride,
                                              int32_t max_blocks, const int32_t* ctx, int32_t num_tokens,
                                              int32_t num_heads, float scale, int32_t num_kv_splits, float* workspace,
                                              int64_t workspace_floats, const uint8_t* empty, void* out,
                                              int64_t out_stride_t, int64_t out_stride_h, float* lse,
                                              int* error_flag, void* stream) {
  if (page != kHdPage) {
    set_error("per-head history: page size %d unsupported (16)", page);
    return kStatusInvalid;
  }
  if (num_tokens < 0 || num_heads < 1 || kv_heads < 1 || num_heads % kv_heads || num_kv_splits < 1 ||
      !ctx || !block_table || !lse || !out) {
    set_error("per-head history: H must be a multiple of kvH, splits >= 1, ctx / table / out / lse set");
    return kStatusInvalid;
  }
  if (key_width % 8 || value_width % 8 || value_width < 8 || value_width > key_width ||
      value_width > kHdMaxCols * kHdThreads || key_width > 1024) {
    set_error("per-head history: widths must be multiples of 8 with value <= key, value <= %d, key <= 1024",
              kHdMaxCols * kHdThreads);
    return kStatusInvalid;
  }
  if ((reinterpret_cast<uintptr_t>(cache) % 16) || (cache_stride_block % 8) || (cache_stride_head % 8) ||
      (cache_stride_row % 8) || cache_stride_row < key_width) {
    set_error("per-head history: the cache needs 16-byte aligned rows (strides multiples of 8 elements)");
    return kStatusInvalid;
  }
  const int64_t need = static_cast<int64_t>(num_tokens) * num_heads * num_kv_splits * (value_width + 1);
  if (need > workspace_floats) {
    set_error("S6 workspace overflow: need %lld floats, have %lld", static_cast<long long>(need),
              static_cast<long long>(workspace_floats));
    return kStatusOverflow;
  }
  if (num_tokens == 0) return kStatusOk;
  HeadsParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.cache = static_cast<const __nv_bfloat16*>(cache);
  p.c_sb = cache_stride_block;
  p.c_sh = cache_stride_head;
  p.c_sr = cache_stride_row;
  p.nb = num_blocks;
  p.bt = block_table;
  p.bt_st = block_table_stride;
  p.max_blocks = max_blocks;
  p.ctx = ctx;
  p.T = num_tokens;
  p.H = num_heads;
  p.kvH = kv_heads;
  p.Lk = key_width;
  p.Lv = value_width;
  p.splits = num_kv_splits;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.ws = workspace;
  p.err = error_flag;
  const int smem = kHdStages * kHdPage * key_width * 2 + (key_width + kHdPage) * 4;
  static unsigned attr_mask = 0;
  ensure_smem_limit(history_heads_split_kernel, kHdStages * kHdPage * 1024 * 2 + (1024 + kHdPage) * 4, attr_mask);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ctas = static_cast<int64_t>(num_tokens) * num_heads * num_kv_splits;
  if (ctas > 0x7fffffff) {
    set_error("per-head history: too many (token, head, split) programs");
    return kStatusInvalid;
  }
  history_heads_split_kernel<<<static_cast<unsigned>(ctas), kHdThreads, smem, s>>>(p);
  int rc = cuda_status(cudaGetLastError(), "history_heads_split_kernel launch");
  if (rc) return rc;
  history_heads_reduce_kernel<<<num_tokens * num_heads, kHdThreads, 0, s>>>(
      workspace, num_heads, num_tokens, num_kv_splits, value_width, empty, static_cast<__nv_bfloat16*>(out),
      out_stride_t, out_stride_h, lse);
  return cuda_status(cudaGetLastError(), "history_heads_reduce_kernel launch");
}
