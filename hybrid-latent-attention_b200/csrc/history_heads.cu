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
// at ~1 flop per byte, an HBM stream; the heads-as-M tiling of the MQA reader does not apply.
//  * Work: a "row" is one (token, head) pair; its pages are the ceil(ctx / 16) pages of its KV head.
//    The grid (SMs x resident CTAs, each CTA one warp) splits the flattened (row, page) space evenly
//    (stream-K), so the step has no tail wave whatever the row count and lengths.  CTA c writes the
//    partial of each row it touched to slot c + row, and CTA 0 records every row's slot range.  A
//    call with num_kv_splits == 1, or a workspace too small for that, runs num_kv_splits CTAs per row
//    over fixed page ranges instead.
//  * Loads: one TMA request per page.  A 5-D tensor map (columns, 16 rows, slabs, kv head, block)
//    lands a page of one KV head as slabs of [16 rows][slab bytes], swizzled so that ldmatrix over 8
//    consecutive keys of one column chunk touches 8 distinct bank groups: MODE 64 (key width a
//    multiple of 32) has Lk / 32 slabs of 64 bytes (64-byte swizzle), MODE 32 Lk / 16 slabs of 32
//    bytes (32-byte swizzle).  The stages form a two-deep per-warp ring with one mbarrier each
//    (kHdStages).  The last page of a row has its rows past ctx zeroed in shared memory after it lands
//    (they may hold anything, +inf or NaN included).  Measured against per-row bulk copies into padded
//    rows: equal at 1152-byte rows, 1.3x faster at 320-byte rows; 128-byte slabs cost more
//    instructions per page and ran slower.
//  * Arithmetic: mma.sync m16n8k16 with the vector (q, then p) replicated into all 8 columns of the
//    N = 8 operand, so a 16-key page costs Lk/16 + Lv/16 tensor instructions, no per-element
//    conversions and no predicated operand loads:
//      scores   S[16 keys]  = K_tile (A: 16 keys x 16 columns) . q (B)
//      values   O^T[Lv]    += V_tile^T (A: ldmatrix.trans, 16 value columns x 16 keys) . p (B)
//    Per-lane operand offsets are computed once.  The online softmax runs on the 16 scores (every lane
//    holds keys g8 and g8 + 8), with a lazy running max (kHdLazyMax).
//  * Partials: [slot][Lv + 1] (normalised output, natural-log lse) in the caller's workspace, which is
//    sized like the reference's attn_logits [T, H, splits, Lv + 1]; a second kernel merges each row's
//    slots.
#include <mutex>

#include "../../include/hla_s6.h"
#include "common.cuh"
#include "hla_s6_internal.h"

namespace hla {

constexpr int kHdPage = 16, kHdThreads = 128;   // kHdThreads: the reduce kernel's block
constexpr int kHdMaxLv = 512, kHdMaxCols = kHdMaxLv / kHdThreads;

struct HeadsParams {
  const __nv_bfloat16* q;  // [T, H, Lk]
  int64_t q_st, q_sh;
  int64_t nb;
  const int32_t* bt;
  int64_t bt_st;
  int max_blocks;
  const int32_t* ctx;
  int T, H, kvH, Lk, Lv;
  int stream;     // 1: stream-K over the flattened (row, page) space; 0: `splits` CTAs per row
  int splits;
  int grid;       // CTAs launched (stream mode)
  int slots_cap;  // partial slots the workspace holds
  float scale_log2;
  float* ws;      // [slots_cap][Lv + 1]
  int2* meta;     // [T * H] slot range of each row (stream mode)
  int* err;
  uint64_t wait_ns;  // bound of every mbarrier wait (device ns)
};

// Stages of the per-warp ring: one page being read while the next lands.  A deeper ring holds more
// bytes in flight per warp but fewer warps per SM; the warps are what the stream needs (measured at
// B = 64, ctx 8192, 16 heads: 93% of the HBM copy peak with 2 stages at 320-byte rows, 89% with 3, 85%
// with 4).
constexpr int kHdStages = 2;
inline int heads_smem_bytes(int Lk) { return 512 + kHdStages * kHdPage * Lk * 2 + Lk * 2 + 64; }

__device__ __forceinline__ int heads_pages(const int32_t* ctx, int t) {
  return (max(ctx[t], 0) + kHdPage - 1) / kHdPage;
}

// Shared-memory offset of 16-byte column chunk `col / 8` of key row `key` in a staged page (`col` a
// multiple of 8).  MODE 64 (key width a multiple of 32): slabs of [16 rows][64 B], 64-byte swizzle
// (chunk bits 4-5 XOR address bits 7-8 = (key / 2) % 4).  MODE 32: slabs of [16][32 B], 32-byte swizzle
// (bit 4 XOR bit 7 = (key / 4) % 2).  Stages are aligned to 512 bytes, the longer swizzle period.
template <int MODE>
__device__ __forceinline__ uint32_t heads_tile_off(int key, int col) {
  if (MODE == 64)
    return static_cast<uint32_t>((col >> 5) * (kHdPage * 64) + key * 64 + ((((col & 31) >> 3) ^ ((key >> 1) & 3)) << 4));
  return static_cast<uint32_t>((col >> 4) * (kHdPage * 32) + key * 32 + ((((col & 15) >> 3) ^ ((key >> 2) & 1)) << 4));
}

// The running max moves only when a page's max exceeds it by more than this (log2 units): the
// exponentials stay below 2^8, and the rescale of the accumulators is skipped on almost every page.
constexpr float kHdLazyMax = 8.f;

// D = A . B with only D's rows g8 / g8 + 8 of column 2 * c4 kept (B's columns are all equal here).
__device__ __forceinline__ void mma_col0(float& c0, float& c2, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "{\n"
      ".reg .f32 d1, d3;\n"
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,d1,%1,d3}, {%2,%3,%4,%5}, {%6,%7}, {%0,%8,%1,%8};\n"
      "}\n"
      : "+f"(c0), "+f"(c2)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ int64_t warp_incl_scan(int64_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// VT = Lv / 16 value tiles; MODE = 64 or 32 (the slab width in bytes, heads_tile_off).
//
// Every mma here has one useful "column": q (scores) or p (values).  It is replicated into all 8
// columns of the B operand, so every lane loads the same fragment words (broadcast, no predicates) and
// every lane ends up holding the scores of keys g8 and g8 + 8.
template <int VT, int MODE>
__global__ void __launch_bounds__(32) history_heads_split_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                 const HeadsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 511) & ~uintptr_t(511));
  const int lane = threadIdx.x, g8 = lane >> 2, c4 = lane & 3;
  const int T = p.T, H = p.H, grp = H / p.kvH, Lk = p.Lk, Lv = p.Lv;
  constexpr int S = kHdStages;
  const uint32_t stage_bytes = static_cast<uint32_t>(kHdPage * Lk * 2);
  // q of the current row in B-fragment order: per 16 columns k0, word pair c4 = {q[k0+2c4 .. +1], q[k0+8+2c4 .. +1]}
  uint2* qf = reinterpret_cast<uint2*>(smem + S * stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes + Lk * 2);   // [S] page landed
  const uint32_t tiles = smem_u32(smem), qbase = smem_u32(qf);

  // ---- this CTA's pages: `count` pages starting at page lp of row (t, h); row r's partial goes to
  //      slot slot0 + r (stream mode) or slot0 (split mode)
  int t = 0, h = 0, lp = 0;
  int64_t count = 0;
  int slot0 = blockIdx.x, slot_row = 0;
  if (p.stream) {
    int64_t P = 0;
    for (int b = 0; b < T; b += 32) {
      const int i = b + lane;
      P += __shfl_sync(0xffffffffu, warp_incl_scan(i < T ? heads_pages(p.ctx, i) : 0, lane), 31);
    }
    P *= H;
    const int64_t G = P < p.grid ? P : static_cast<int64_t>(p.grid);
    if (blockIdx.x == 0) {
      // every row's slot range [owner(first page) + r, owner(last page) + r + 1)
      int64_t carry = 0;
      for (int b = 0; b < T; b += 32) {
        const int i = b + lane;
        const int np = i < T ? heads_pages(p.ctx, i) : 0;
        const int64_t v = static_cast<int64_t>(np) * H, inc = warp_incl_scan(v, lane), start = carry + inc - v;
        if (i < T) {
          for (int hh = 0; hh < H; ++hh) {
            const int r = i * H + hh;
            int2 m = make_int2(0, 0);
            if (np > 0) {
              const int64_t a = start + static_cast<int64_t>(hh) * np, e = a + np;
              m = make_int2(static_cast<int>(stream_owner(a, P, G)) + r, static_cast<int>(stream_owner(e - 1, P, G)) + r + 1);
            }
            p.meta[r] = m;
          }
        }
        carry += __shfl_sync(0xffffffffu, inc, 31);
      }
    }
    if (static_cast<int64_t>(blockIdx.x) >= G) return;
    const int64_t p0 = stream_start(blockIdx.x, P, G);
    count = stream_start(blockIdx.x + 1, P, G) - p0;
    slot_row = 1;
    // the token whose pages hold p0
    int64_t carry = 0;
    for (int b = 0; b < T; b += 32) {
      const int i = b + lane;
      const int64_t v = i < T ? static_cast<int64_t>(heads_pages(p.ctx, i)) * H : 0, inc = warp_incl_scan(v, lane);
      const unsigned hit = __ballot_sync(0xffffffffu, v > 0 && carry + inc > p0);
      if (hit) {
        const int L = __ffs(hit) - 1;
        t = b + L;
        const int64_t off = p0 - (carry + __shfl_sync(0xffffffffu, inc - v, L));
        const int np = heads_pages(p.ctx, t);
        h = static_cast<int>(off / np);
        lp = static_cast<int>(off % np);
        break;
      }
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
  } else {
    const int r = blockIdx.x / p.splits, s = blockIdx.x % p.splits;
    t = r / H;
    h = r % H;
    const int np = heads_pages(p.ctx, t), per = (np + p.splits - 1) / p.splits;
    lp = s * per;
    count = max(0, min(np, lp + per) - lp);
    if (count == 0) {  // nothing to read in this split
      if (slot0 < p.slots_cap) {
        float* out = p.ws + static_cast<int64_t>(slot0) * (Lv + 1);
        for (int c = lane; c < Lv; c += 32) out[c] = 0.f;
        if (lane == 0) out[Lv] = -INFINITY;
      }
      return;
    }
  }

  if (lane == 0) {
    for (int s2 = 0; s2 < S; ++s2) mbar_init(&full[s2], 1);
    fence_barrier_init();
    prefetch_tmap(&tmap);
  }
  __syncwarp();

  // first page of the row after (tt, hh): the next head, else the next token with pages
  auto next_row = [&](int& tt, int& hh, int& ll, int& np) {
    ll = 0;
    if (++hh < H) return;
    hh = 0;
    do {
      ++tt;
    } while (tt < T && (np = heads_pages(p.ctx, tt)) == 0);
  };
  // ---- producer cursor (token, head, page, pages of the token) and its block-id cache: 32 table
  //      entries per coalesced load, broadcast by shuffle
  int pt = t, ph = h, plp = lp, pnp = heads_pages(p.ctx, t);
  int ids_t = -1, ids_chunk = -1, ids = -1;
  auto issue = [&](int stage) {
    const int chunk = plp >> 5;
    if (pt != ids_t || chunk != ids_chunk) {
      ids_t = pt;
      ids_chunk = chunk;
      const int j = (chunk << 5) + lane;
      ids = (j < pnp && j < p.max_blocks) ? p.bt[static_cast<int64_t>(pt) * p.bt_st + j] : -1;
    }
    const int blk = __shfl_sync(0xffffffffu, ids, plp & 31);
    const bool ok = blk >= 0 && blk < p.nb;
    uint8_t* dst = smem + stage * stage_bytes;
    // generic-proxy accesses of this stage (the previous page's reads, zero fills) precede the copy
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      if (!ok) record_error(p.err, kErrSlots);
      mbar_arrive_expect_tx(&full[stage], ok ? stage_bytes : 0u);
      if (ok) tma_load_5d(dst, &tmap, &full[stage], 0, 0, 0, ph / grp, blk);
    }
    if (!ok) {  // a block id outside the cache reads as zeros
      for (uint32_t c = lane; c < stage_bytes / 16; c += 32) reinterpret_cast<uint4*>(dst)[c] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (++plp == pnp) next_row(pt, ph, plp, pnp);
  };
  auto load_q = [&]() {
    const uint4* qr = reinterpret_cast<const uint4*>(p.q + static_cast<int64_t>(t) * p.q_st +
                                                     static_cast<int64_t>(h) * p.q_sh);
    for (int g = lane; g < Lk / 16; g += 32) {
      const uint4 lo = qr[2 * g], hi = qr[2 * g + 1];  // columns 16g .. +7 and 16g + 8 .. +15
      reinterpret_cast<uint4*>(qf + 4 * g)[0] = make_uint4(lo.x, hi.x, lo.y, hi.y);
      reinterpret_cast<uint4*>(qf + 4 * g)[1] = make_uint4(lo.z, hi.z, lo.w, hi.w);
    }
    __syncwarp();
  };

  // per-lane shared-memory offsets of the two operand tiles (page-independent)
  const int skey = lane & 15, sc = lane >> 4;                                  // scores: A rows = keys
  const int vkey = (lane & 7) + ((lane >> 4) << 3), vc = (lane >> 3) & 1;     // values: A^T rows = keys
  uint32_t so0, so1, vo0, vo1;
  if (MODE == 64) {
    so0 = skey * 64 + ((sc ^ ((skey >> 1) & 3)) << 4);         // even 16-column step of a slab
    so1 = skey * 64 + (((sc + 2) ^ ((skey >> 1) & 3)) << 4);   // odd step
    vo0 = vkey * 64 + ((vc ^ ((vkey >> 1) & 3)) << 4);
    vo1 = vkey * 64 + (((vc + 2) ^ ((vkey >> 1) & 3)) << 4);
  } else {
    so0 = so1 = skey * 32 + ((sc ^ ((skey >> 2) & 1)) << 4);
    vo0 = vo1 = vkey * 32 + ((vc ^ ((vkey >> 2) & 1)) << 4);
  }
  const int ksteps = Lk / 16;

  int64_t issued = 0;
  for (; issued < S - 1 && issued < count; ++issued) issue(static_cast<int>(issued % S));
  load_q();

  int np = heads_pages(p.ctx, t), n = max(p.ctx[t], 0);
  float m = -INFINITY, l = 0.f;
  float oc0[VT], oc2[VT];  // O^T rows g8 and g8 + 8 of value tile vt (column 2 c4; equal in every c4)
#pragma unroll
  for (int i = 0; i < VT; ++i) oc0[i] = oc2[i] = 0.f;

  for (int64_t it = 0; it < count; ++it) {
    if (issued < count) {
      issue(static_cast<int>(issued % S));
      ++issued;
    }
    const int stage = static_cast<int>(it % S);
    const bool landed = __all_sync(0xffffffffu, mbar_wait(&full[stage], static_cast<uint32_t>((it / S) & 1), p.wait_ns));
    if (!landed) {
      // give up, but not before the copies already issued into this CTA's shared memory have
      // completed (bounded waits)
      if (lane == 0) record_error(p.err, kErrWaitFull);
      for (int64_t q2 = it + 1; q2 < issued; ++q2)
        mbar_wait(&full[q2 % S], static_cast<uint32_t>((q2 / S) & 1), p.wait_ns);
      return;
    }
    const uint32_t tb = tiles + stage * stage_bytes;
    const int valid = min(kHdPage, n - lp * kHdPage);
    if (valid < kHdPage) {
      // rows past ctx: zero them (the swizzle keeps each row's chunks inside its own slab row)
      uint8_t* st = smem + stage * stage_bytes;
      const int per_row = Lk / 8, total = (kHdPage - valid) * per_row;
      for (int c = lane; c < total; c += 32) {
        const int key = valid + c / per_row, col = (c % per_row) * 8;
        *reinterpret_cast<uint4*>(st + heads_tile_off<MODE>(key, col)) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    __syncwarp();
    // ---- scores of the 16 keys (every lane: keys g8 and g8 + 8)
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
    if (MODE == 64) {
      for (int i = 0; i < ksteps; i += 2) {  // one 64-byte slab = two 16-column steps
        const uint32_t slab = tb + (i >> 1) * (kHdPage * 64);
        uint32_t a[4], b[2];
        ldsm_x4(slab + so0, a[0], a[1], a[2], a[3]);
        asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(b[0]), "=r"(b[1]) : "r"(qbase + i * 32 + c4 * 8));
        mma_bf16_16816(sacc, a, b[0], b[1]);
        ldsm_x4(slab + so1, a[0], a[1], a[2], a[3]);
        asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(b[0]), "=r"(b[1]) : "r"(qbase + i * 32 + 32 + c4 * 8));
        mma_bf16_16816(sacc, a, b[0], b[1]);
      }
    } else {
      for (int i = 0; i < ksteps; ++i) {
        uint32_t a[4], b[2];
        ldsm_x4(tb + i * (kHdPage * 32) + so0, a[0], a[1], a[2], a[3]);
        asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(b[0]), "=r"(b[1]) : "r"(qbase + i * 32 + c4 * 8));
        mma_bf16_16816(sacc, a, b[0], b[1]);
      }
    }
    const float s0 = g8 < valid ? sacc[0] * p.scale_log2 : -INFINITY;
    const float s1 = g8 + 8 < valid ? sacc[2] * p.scale_log2 : -INFINITY;
    // ---- online softmax over the page (lazy max: see kHdLazyMax)
    float tm = fmaxf(s0, s1);
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 4));
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 8));
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 16));
    if (tm > m + kHdLazyMax) {  // warp-uniform; always taken on a row's first page (m = -inf)
      const float alpha = exp2f(m - tm);
      l *= alpha;
#pragma unroll
      for (int vt = 0; vt < VT; ++vt) {
        oc0[vt] *= alpha;
        oc2[vt] *= alpha;
      }
      m = tm;
    }
    const float p0 = exp2f(s0 - m), p1 = exp2f(s1 - m);  // 0 for masked keys
    float ps = p0 + p1;
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
    l += ps;
    // ---- P as the B operand (every column): lane c4 takes keys 2c4, 2c4 + 1, 2c4 + 8, 2c4 + 9
    //      (key j < 8 lives in lanes 4j .. 4j + 3 as p0, key j + 8 there as p1)
    const float pa = __shfl_sync(0xffffffffu, p0, 8 * c4), pb = __shfl_sync(0xffffffffu, p0, 8 * c4 + 4);
    const float pc = __shfl_sync(0xffffffffu, p1, 8 * c4), pd = __shfl_sync(0xffffffffu, p1, 8 * c4 + 4);
    const uint32_t b0 = pack_bf16(pa, pb), b1 = pack_bf16(pc, pd);
    // ---- O^T += V^T . P
#pragma unroll
    for (int vt = 0; vt < VT; ++vt) {
      uint32_t a[4];
      const uint32_t off = MODE == 64 ? (vt >> 1) * (kHdPage * 64) + ((vt & 1) ? vo1 : vo0) : vt * (kHdPage * 32) + vo0;
      ldsm_x4_t(tb + off, a[0], a[1], a[2], a[3]);
      mma_col0(oc0[vt], oc2[vt], a, b0, b1);
    }
    __syncwarp();  // the stage is consumed before the next copy overwrites it

    // ---- end of this CTA's part of the row: write its partial, move to the next row
    const bool last = it + 1 == count;
    if (++lp == np || last) {
      const int slot = slot0 + slot_row * (t * H + h);
      if (slot < p.slots_cap) {
        float* out = p.ws + static_cast<int64_t>(slot) * (Lv + 1);
        const float inv = l > 0.f ? 1.f / l : 0.f;
        if (c4 == 0) {
#pragma unroll
          for (int vt = 0; vt < VT; ++vt) {
            out[vt * 16 + g8] = oc0[vt] * inv;
            out[vt * 16 + g8 + 8] = oc2[vt] * inv;
          }
        }
        if (lane == 0) out[Lv] = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
      } else if (lane == 0) {
        record_error(p.err, kErrSlots);
      }
      if (!last) {
        m = -INFINITY;
        l = 0.f;
#pragma unroll
        for (int i = 0; i < VT; ++i) oc0[i] = oc2[i] = 0.f;
        next_row(t, h, lp, np);
        n = max(p.ctx[t], 0);
        load_q();
      }
    }
  }
}

// Merge of a (token, head)'s partial slots -> o (bf16, [T, H, Lv] strided) and lse [H, T].  The slots
// are meta[row] (stream mode) or row * splits .. + splits.
__global__ void __launch_bounds__(kHdThreads) history_heads_reduce_kernel(const float* __restrict__ ws,
                                                                          const int2* __restrict__ meta, int splits,
                                                                          int H, int T, int Lv,
                                                                          const uint8_t* __restrict__ empty,
                                                                          __nv_bfloat16* __restrict__ out,
                                                                          int64_t o_st, int64_t o_sh,
                                                                          float* __restrict__ lse) {
  const int row = blockIdx.x, t = row / H, h = row % H, tid = threadIdx.x;
  int lo = row * splits, hi = lo + splits;
  if (meta) {
    const int2 m = meta[row];
    lo = m.x;
    hi = m.y;
  }
  float mx = -INFINITY;
  for (int s = lo; s < hi; ++s) mx = fmaxf(mx, ws[static_cast<int64_t>(s) * (Lv + 1) + Lv]);
  const bool is_empty = (empty && empty[t]) || mx == -INFINITY;
  float wsum = 0.f;
  float acc[kHdMaxCols] = {0.f, 0.f, 0.f, 0.f};
  if (!is_empty) {
    for (int s = lo; s < hi; ++s) {
      const float* part = ws + static_cast<int64_t>(s) * (Lv + 1);
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

// Resident CTAs per SM of one kernel instance at a shared-memory size (cached per device).
template <int VT, int MODE>
static int heads_occupancy(int smem) {
  static std::mutex mu;
  static int cached_smem[32] = {0}, cached_n[32] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 31;
  std::lock_guard<std::mutex> lock(mu);
  if (cached_smem[dev] != smem || cached_n[dev] < 1) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, history_heads_split_kernel<VT, MODE>, 32, smem) !=
            cudaSuccess ||
        n < 1)
      return 1;
    cached_smem[dev] = smem;
    cached_n[dev] = n;
  }
  return cached_n[dev];
}

template <int VT, int MODE>
static int launch_heads(const CUtensorMap& tmap, HeadsParams& p, int64_t ws_floats, cudaStream_t s) {
  static unsigned attr_mask = 0;
  ensure_smem_limit(history_heads_split_kernel<VT, MODE>, heads_smem_bytes(1024), attr_mask);
  const int smem = heads_smem_bytes(p.Lk);
  const int64_t rows = static_cast<int64_t>(p.T) * p.H;
  // stream mode: slots [slots_cap][Lv + 1], then meta [rows] int2 (8-byte aligned)
  const int64_t stream_cap = (ws_floats - 2 * rows - 1) / (p.Lv + 1);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t g = std::min<int64_t>(static_cast<int64_t>(sms) * heads_occupancy<VT, MODE>(smem),
                                      stream_cap - rows + 1);
  int64_t ctas;
  if (p.splits >= 2 && g >= 1 && rows <= (int64_t(1) << 24)) {
    p.stream = 1;
    p.grid = static_cast<int>(g);
    p.slots_cap = static_cast<int>(stream_cap);
    uintptr_t m = reinterpret_cast<uintptr_t>(p.ws + stream_cap * (p.Lv + 1));
    p.meta = reinterpret_cast<int2*>((m + 7) & ~uintptr_t(7));
    ctas = g;
  } else {
    p.stream = 0;
    p.grid = 0;
    p.slots_cap = static_cast<int>(rows * p.splits);
    p.meta = nullptr;
    ctas = rows * p.splits;
  }
  if (ctas > 0x7fffffff) {
    set_error("per-head history: too many (token, head, split) programs");
    return kStatusInvalid;
  }
  history_heads_split_kernel<VT, MODE><<<static_cast<unsigned>(ctas), 32, smem, s>>>(tmap, p);
  return cuda_status(cudaGetLastError(), "history_heads_split_kernel launch");
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
  if (reinterpret_cast<uintptr_t>(q) % 16 || q_stride_t % 8 || q_stride_h % 8) {
    set_error("per-head history: q rows must be 16-byte aligned (strides multiples of 8 elements)");
    return kStatusInvalid;
  }
  const int64_t need = static_cast<int64_t>(num_tokens) * num_heads * num_kv_splits * (value_width + 1);
  if (need > workspace_floats) {
    set_error("S6 workspace overflow: need %lld floats, have %lld", static_cast<long long>(need),
              static_cast<long long>(workspace_floats));
    return kStatusOverflow;
  }
  if (num_tokens == 0) return kStatusOk;
  // MODE 64: 32-column slabs (64-byte swizzle) when the key width allows, else 16-column slabs
  const int mode = key_width % 32 == 0 ? 64 : 32;
  CUtensorMap tmap;
  int rc = heads_cache_tmap(&tmap, cache, num_blocks, kv_heads, cache_stride_block, cache_stride_head,
                            cache_stride_row, mode / 2, key_width / (mode / 2));
  if (rc) return rc;
  HeadsParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
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
  p.wait_ns = wait_limit_ns();
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
#define HLA_HEADS(VT)                                                                               \
  rc = mode == 64 ? launch_heads<VT, 64>(tmap, p, workspace_floats, s) : launch_heads<VT, 32>(tmap, p, workspace_floats, s)
  switch (value_width / 16) {
    case 4: HLA_HEADS(4); break;
    case 8: HLA_HEADS(8); break;
    case 16: HLA_HEADS(16); break;
    case 32: HLA_HEADS(32); break;
    default: set_error("per-head history: value width %d unsupported (64, 128, 256, 512)", value_width);
      return kStatusInvalid;
  }
#undef HLA_HEADS
  if (rc) return rc;
  history_heads_reduce_kernel<<<num_tokens * num_heads, kHdThreads, 0, s>>>(
      workspace, p.meta, num_kv_splits, num_heads, num_tokens, value_width, empty, static_cast<__nv_bfloat16*>(out),
      out_stride_t, out_stride_h, lse);
  return cuda_status(cudaGetLastError(), "history_heads_reduce_kernel launch");
}
