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
// at ~1 flop per byte, an HBM stream; the heads-as-M tiling of the MQA reader does not apply.  Each
// (token, head, split) is one independent warp (a 32-thread CTA, many resident per SM): a ring of
// shared-memory stages holds its pages (16 rows x Lk, rows padded by 16 bytes so ldmatrix is
// conflict-free), each row fetched by one bulk copy (cp.async.bulk, completion counted on the
// stage's mbarrier) - 16 requests per page, where 16-byte cp.async would need Lk / 8 per row and
// exhaust the SM's outstanding-request capacity long before HBM does; rows past ctx are zeroed.  The arithmetic runs on mma.sync m16n8k16 with the vector
// as the N = 8 operand's first column, so a 16-key page costs Lk/16 + Lv/16 tensor instructions and
// no per-element conversions:
//   scores   S[16 keys]  = K_tile (A: 16 keys x 16 columns) . q (B column 0)
//   values   O^T[Lv]    += V_tile^T (A: ldmatrix.trans, 16 value columns x 16 keys) . p (B column 0)
// The online softmax runs on the 16 scores (lanes with c4 = 0 hold two each).  The normalised partial
// and its lse go to the workspace [T, H, splits, Lv + 1] (the reference's attn_logits layout); a second
// kernel merges the splits.
#include "../../include/hla_s6.h"
#include "common.cuh"
#include "hla_s6_internal.h"

namespace hla {

constexpr int kHdPage = 16, kHdThreads = 128;   // kHdThreads: the reduce kernel's block
constexpr int kHdMaxLv = 512, kHdMaxCols = kHdMaxLv / kHdThreads;

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

// Stages of the per-warp ring for a row width (shared memory per warp-CTA stays under ~40 KB).
__host__ __device__ inline int heads_stages(int Lk) { return Lk <= 256 ? 4 : (Lk <= 512 ? 3 : 2); }
__host__ __device__ inline int heads_row_elems(int Lk) { return Lk + 8; }   // +16 B per row
inline int heads_smem_bytes(int Lk) { return 64 + (heads_stages(Lk) * kHdPage * heads_row_elems(Lk) + Lk) * 2; }

// One contiguous global -> shared copy by the bulk-copy engine (no multicast), completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// D = A . B with only D's column 0 kept (rows g8 and g8 + 8 in the c4 = 0 lanes): the other two
// accumulators start at zero and are dropped.
__device__ __forceinline__ void mma_col0(float& c0, float& c2, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "{\n"
      ".reg .f32 d1, d3;\n"
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,d1,%1,d3}, {%2,%3,%4,%5}, {%6,%7}, {%0,%8,%1,%8};\n"
      "}\n"
      : "+f"(c0), "+f"(c2)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// VT = Lv / 16 value tiles.
template <int VT>
__global__ void __launch_bounds__(32, 1) history_heads_split_kernel(const HeadsParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int lane = threadIdx.x, g8 = lane >> 2, c4 = lane & 3;
  const int split = blockIdx.x % p.splits;
  const int row = blockIdx.x / p.splits;  // t * H + h
  const int t = row / p.H, h = row % p.H;
  const int kvh = h / (p.H / p.kvH);
  const int Lk = p.Lk, Lv = p.Lv, lk8 = Lk / 8, RE = heads_row_elems(Lk), S = heads_stages(Lk);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);                       // [S] page landed
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem_raw + 64);          // [Lk]
  __nv_bfloat16* tiles = qs + Lk;                                               // [S][16][RE]
  float* out = p.ws + (static_cast<int64_t>(row) * p.splits + split) * (Lv + 1);

  const int n = max(p.ctx[t], 0);
  const int pages = (n + kHdPage - 1) / kHdPage;
  const int per = (pages + p.splits - 1) / p.splits;
  const int pg0 = split * per, pg1 = min(pages, pg0 + per);
  if (pg0 >= pg1) {  // nothing to read in this split
    for (int c = lane; c < Lv; c += 32) out[c] = 0.f;
    if (lane == 0) out[Lv] = -INFINITY;
    return;
  }
  {
    const uint4* qr = reinterpret_cast<const uint4*>(p.q + static_cast<int64_t>(t) * p.q_st +
                                                     static_cast<int64_t>(h) * p.q_sh);
    for (int c = lane; c < lk8; c += 32) reinterpret_cast<uint4*>(qs)[c] = qr[c];
  }

  // the split's block ids, 32 at a time (one coalesced load per 32 pages; pages are requested in
  // increasing order), broadcast by shuffle so no page waits on its own table read
  int ids_chunk = -1, ids = -1;
  auto block_of = [&](int lp) -> int {
    const int idx = lp - pg0, chunk = idx >> 5;
    if (chunk != ids_chunk) {
      ids_chunk = chunk;
      const int j = pg0 + (chunk << 5) + lane;
      ids = (j < pg1 && j < p.max_blocks) ? p.bt[static_cast<int64_t>(t) * p.bt_st + j] : -1;
    }
    return __shfl_sync(0xffffffffu, ids, idx & 31);
  };
  const uint32_t row_bytes = static_cast<uint32_t>(Lk) * 2;
  auto load_page = [&](int lp, int stage) {
    int blk = block_of(lp);
    if (blk < 0 || blk >= p.nb) {
      if (lane == 0) record_error(p.err, kErrSlots);
      blk = -1;
    }
    const int valid = blk < 0 ? 0 : min(kHdPage, n - lp * kHdPage);
    __nv_bfloat16* dst = tiles + stage * kHdPage * RE;
    // generic-proxy accesses of this stage (the previous page's reads, zero fills) precede the copies
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(valid) * row_bytes);
    __syncwarp();
    if (lane < valid) {
      const __nv_bfloat16* src = p.cache + static_cast<int64_t>(blk) * p.c_sb + static_cast<int64_t>(kvh) * p.c_sh +
                                 static_cast<int64_t>(lane) * p.c_sr;
      bulk_g2s(dst + lane * RE, src, row_bytes, &full[stage]);
    } else if (lane < kHdPage) {
      uint4* z = reinterpret_cast<uint4*>(dst + lane * RE);  // rows past ctx read as zeros
      for (int c = 0; c < lk8; ++c) z[c] = make_uint4(0u, 0u, 0u, 0u);
    }
  };

  if (lane == 0) {
    for (int s2 = 0; s2 < S; ++s2) mbar_init(&full[s2], 1);
    fence_barrier_init();
  }
  __syncwarp();
  for (int s2 = 0; s2 < S - 1; ++s2)
    if (pg0 + s2 < pg1) load_page(pg0 + s2, s2);
  __syncwarp();

  float m = -INFINITY, l = 0.f;
  float oc0[VT], oc2[VT];  // O^T rows g8 and g8 + 8 of value tile vt (meaningful in c4 = 0 lanes)
#pragma unroll
  for (int i = 0; i < VT; ++i) oc0[i] = oc2[i] = 0.f;
  const uint32_t qbase = smem_u32(qs);

  for (int lp = pg0, it = 0; lp < pg1; ++lp, ++it) {
    const int nxt = lp + S - 1;
    if (nxt < pg1) load_page(nxt, (it + S - 1) % S);
    const bool landed = __all_sync(0xffffffffu, mbar_wait(&full[it % S], (it / S) & 1));
    if (!landed) {
      // give up on this split, but not before the copies already issued into this CTA's shared
      // memory have completed (bounded waits)
      if (lane == 0) record_error(p.err, kErrWaitFull);
      for (int q = it + 1, lq = lp + 1; lq < pg1 && q <= it + S - 1; ++q, ++lq) mbar_wait(&full[q % S], (q / S) & 1);
      break;
    }
    __syncwarp();
    const uint32_t tb = smem_u32(tiles + (it % S) * kHdPage * RE);
    const int valid = min(kHdPage, n - lp * kHdPage);
    // ---- scores of the 16 keys
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < Lk; k0 += 16) {
      uint32_t a[4];
      ldsm_x4(tb + (((lane & 15) * RE + k0 + ((lane >> 4) << 3)) << 1), a[0], a[1], a[2], a[3]);
      uint32_t b0 = 0u, b1 = 0u;
      if (g8 == 0) {
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b0) : "r"(qbase + ((k0 + 2 * c4) << 1)));
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b1) : "r"(qbase + ((k0 + 8 + 2 * c4) << 1)));
      }
      mma_bf16_16816(sacc, a, b0, b1);
    }
    const float s0 = (c4 == 0 && g8 < valid) ? sacc[0] * p.scale_log2 : -INFINITY;
    const float s1 = (c4 == 0 && g8 + 8 < valid) ? sacc[2] * p.scale_log2 : -INFINITY;
    // ---- online softmax over the tile
    float tm = fmaxf(s0, s1);
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 4));
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 8));
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 16));
    tm = __shfl_sync(0xffffffffu, tm, 0);
    const float mn = fmaxf(m, tm);  // finite: every visited page has a key below ctx
    const float alpha = exp2f(m - mn);
    const float p0 = exp2f(s0 - mn), p1 = exp2f(s1 - mn);  // 0 for masked keys and c4 != 0 lanes
    float ps = p0 + p1;
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
    ps = __shfl_sync(0xffffffffu, ps, 0);
    l = l * alpha + ps;
    m = mn;
    // ---- P as the B operand's column 0: lane c4 of g8 = 0 takes keys 2c4, 2c4 + 1, 2c4 + 8, 2c4 + 9
    //      (key j < 8 lives in lane 4j as p0, key j + 8 there as p1)
    const float pa = __shfl_sync(0xffffffffu, p0, 8 * c4), pb = __shfl_sync(0xffffffffu, p0, 8 * c4 + 4);
    const float pc = __shfl_sync(0xffffffffu, p1, 8 * c4), pd = __shfl_sync(0xffffffffu, p1, 8 * c4 + 4);
    const uint32_t b0 = g8 == 0 ? pack_bf16(pa, pb) : 0u, b1 = g8 == 0 ? pack_bf16(pc, pd) : 0u;
    // ---- O^T += V^T . P
    const int vkey = (lane & 7) + ((lane >> 4) << 3), vcol = ((lane >> 3) & 1) << 3;
#pragma unroll
    for (int vt = 0; vt < VT; ++vt) {
      oc0[vt] *= alpha;
      oc2[vt] *= alpha;
      uint32_t a[4];
      ldsm_x4_t(tb + ((vkey * RE + vt * 16 + vcol) << 1), a[0], a[1], a[2], a[3]);
      mma_col0(oc0[vt], oc2[vt], a, b0, b1);
    }
    __syncwarp();  // the stage is consumed before the next load overwrites it
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  if (c4 == 0) {
#pragma unroll
    for (int vt = 0; vt < VT; ++vt) {
      out[vt * 16 + g8] = oc0[vt] * inv;
      out[vt * 16 + g8 + 8] = oc2[vt] * inv;
    }
  }
  if (lane == 0) out[Lv] = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
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
  if (key_width % 16 || value_width % 16 || value_width < 16 || value_width > key_width || value_width > kHdMaxLv ||
      key_width > 1024) {
    set_error("per-head history: widths must be multiples of 16 with value <= key, value <= %d, key <= 1024",
              kHdMaxLv);
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
  const int smem = heads_smem_bytes(key_width);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ctas = static_cast<int64_t>(num_tokens) * num_heads * num_kv_splits;
  if (ctas > 0x7fffffff) {
    set_error("per-head history: too many (token, head, split) programs");
    return kStatusInvalid;
  }
#define HLA_HEADS(VT)                                                                                   \
  {                                                                                                    \
    static unsigned attr_mask = 0;                                                                     \
    ensure_smem_limit(history_heads_split_kernel<VT>, heads_smem_bytes(1024), attr_mask);              \
    history_heads_split_kernel<VT><<<static_cast<unsigned>(ctas), 32, smem, s>>>(p);                   \
  }
  switch (value_width / 16) {
    case 4: HLA_HEADS(4); break;
    case 8: HLA_HEADS(8); break;
    case 16: HLA_HEADS(16); break;
    case 32: HLA_HEADS(32); break;
    default: set_error("per-head history: value width %d unsupported (64, 128, 256, 512)", value_width);
      return kStatusInvalid;
  }
#undef HLA_HEADS
  int rc = cuda_status(cudaGetLastError(), "history_heads_split_kernel launch");
  if (rc) return rc;
  history_heads_reduce_kernel<<<num_tokens * num_heads, kHdThreads, 0, s>>>(
      workspace, num_heads, num_tokens, num_kv_splits, value_width, empty, static_cast<__nv_bfloat16*>(out),
      out_stride_t, out_stride_h, lse);
  return cuda_status(cudaGetLastError(), "history_heads_reduce_kernel launch");
}
