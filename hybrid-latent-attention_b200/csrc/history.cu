// Paged latent-history reader of the S6 decode path (split-K attention + split count / workspace).
//
// Reference behaviour: hla/vllm_latent/s6_ops.py:117-161 (history_attention /
// history_attention_kv) and its torch oracle s6_ops.py:204-222 (_history_reference):
// a fully visible softmax of q_lat[T,H,W] over the first ctx[t] rows of an MQA latent cache
// [num_blocks, 1, page, 2W] (row = K | V), paged through a per-token block table.  Only
// block-table columns < ceil(ctx[t] / page) are read.  Empty rows give o = 0, lse = -inf.
//
// B200 design
//  * one producer warp streams whole pages with a 4-D TMA tensor map
//    (64-element inner box, rows, 64-column slabs, blocks) and SWIZZLE_128B into a STAGES-deep
//    shared-memory ring (mbarrier complete_tx); no multicast - every CTA reads its own pages.
//  * NC = W/128 consumer warps each own 128 latent columns.  Heads are the M = 16 dimension
//    of mma.m16n8k16 (the 16 query heads share one KV head), keys are N, columns are K:
//      S_w  = Q[:, cols_w] . K[keys, cols_w]^T   (partial scores, reduced across warps in smem)
//      O_w += P . V[keys, cols_w]                (P reused from the score fragments, FA2 style)
//  * stream-K partition: the grid splits the flattened (row, page) space evenly, so mixed
//    lengths balance across the 148 SMs; each CTA emits one fp32 partial (o, lse) per row
//    segment it touched into the caller's workspace.  CTA c writes row t's partial at slot
//    c + t, and CTA 0 records each row's slot range in `meta`.
//  * tail stealing (the STEAL kernel, for steps with about as many rows as CTAs): the last eighth
//    of every CTA's range goes to a shared pool that CTAs drain once their own part is done, so
//    CTAs slowed by the memory system finish with the others.  Units - a CTA's main part, or a
//    tail - keep fixed partial slots (unit u, row t: slot u + t), so the result does not depend
//    on which CTA ran a unit.
//  * a reduce kernel (the Triton stage-2 equivalent) or the fused decode combine turns the
//    partials into the op outputs.
#include <mutex>

#include "common.cuh"
#include "hla_s6_internal.h"

namespace hla {

struct HistoryParams {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;          // q strides (elements) for token and head; unit last stride
  const int32_t* block_table;  // [T, max_blocks] per token
  int64_t bt_st;
  int32_t max_blocks;          // columns beyond it load as zeros (never read out of the table)
  const int32_t* ctx;          // [T] rows of history to read
  int32_t T, H;
  float scale_log2;            // softmax scale * log2(e)
  float* ws_o;                 // [slots][H][W] normalised partial outputs
  float* ws_lse;               // [slots][H] natural-log partial lse
  int2* meta;                  // [T] slot range per row (stream mode)
  int32_t slots_cap;
  int32_t grid;                // CTAs launched (stream mode)
  int32_t stream_mode;         // 1: stream-K over pages, 0: one CTA per row
  int* err;
  uint64_t wait_ns;            // bound of every mbarrier wait (device ns)
  int64_t num_blocks;          // cache blocks: a table entry outside [0, num_blocks) sets kErrBlock
  // contiguous layout (the HF engines' reader): every row has contig_n keys in K/V [rows, N, W]
  // (tile = PG consecutive keys of the row; two tensor maps, K and V) and a per-key mask
  int32_t contig_n;
  const uint8_t* mask;  // [rows, N], nonzero = visible
  int64_t mask_st;
  // paged stream mode: [0] tail ticket, [1] CTAs done; zero between launches (the last CTA of a
  // launch re-zeroes them).  NULL: every CTA keeps its whole page range (no tail stealing).
  unsigned* steal;
};

template <int W, int PG>
struct HistoryCfg {
  static constexpr int NC = W / 128;                   // consumer warps
  static constexpr int NT = PG / 8;                    // n8 key tiles per page
  static constexpr int SLAB_BYTES = PG * 128;          // one 64-column slab of a page
  static constexpr int PAGE_BYTES = PG * 2 * W * 2;    // K and V of a page, bf16
  static constexpr int STAGES = PAGE_BYTES <= 16384 ? 4 : (PAGE_BYTES <= 32768 ? 3 : 2);
  static constexpr int THREADS = (NC + 1) * 32;
  static constexpr int XBUF_BYTES = 2 * NC * NT * 32 * 16;
  // Resident CTAs per SM the register budget is sized for: two for 512-wide 16-row pages, and for
  // 256-wide pages a bound that keeps registers <= 168, so three 3-warp CTAs fit each SM
  // sub-partition's register file (shared memory also allows three).
  static constexpr int MIN_CTAS = PAGE_BYTES <= 16384 ? 4 : ((STAGES * PAGE_BYTES <= 100 * 1024) ? 2 : 1);
};

__device__ __forceinline__ uint32_t mask_pair(uint32_t v, int key_lo, int valid) {
  if (key_lo >= valid) return 0u;
  if (key_lo + 1 >= valid) return v & 0xffffu;
  return v;
}

// CONTIG: the contiguous-layout front end (fused_history.py:49-54, history_kernels.py:11-33):
// `tmap` covers K [rows, N, W] and `tmap_v` V, both as (64, N, W/64, rows) boxes of PG keys, so a
// tile lands in shared memory exactly as a page of the paged cache does (K slabs, then V slabs);
// rows have p.contig_n keys and a per-key mask instead of a prefix length.
template <int W, int PG, bool CONTIG = false, bool STEAL = false>
__global__ void __launch_bounds__(HistoryCfg<W, PG>::THREADS, HistoryCfg<W, PG>::MIN_CTAS)
    history_split_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap tmap_v,
                         const HistoryParams p) {
  using C = HistoryCfg<W, PG>;
  constexpr int NC = C::NC, NT = C::NT, STAGES = C::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  float4* xbuf = reinterpret_cast<float4*>(smem + STAGES * C::PAGE_BYTES);
  // per stage: row, local page, slot, flags (16-byte aligned: it follows the 16-byte multiples above)
  int4* smeta = reinterpret_cast<int4*>(smem + STAGES * C::PAGE_BYTES + C::XBUF_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(smeta + STAGES);
  uint64_t* empty = full + STAGES;
  uint64_t* mready = empty + STAGES;                   // per stage: its descriptor is written
  int* misc = reinterpret_cast<int*>(mready + STAGES);  // [0]=abort
  int* pref = misc + 4;                                 // [T+1] page prefix (stream mode)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.T;
  int64_t P = 0, G = 1, p0 = 0, p1 = 0;
  int row0 = 0;
  bool steal_on = false;

  if (p.stream_mode) {
    for (int t = tid; t < T; t += blockDim.x) {
      const int c = CONTIG ? p.contig_n : max(p.ctx[t], 0);
      pref[t + 1] = (c + PG - 1) / PG;
    }
    if (tid == 0) pref[0] = 0;
    __syncthreads();
    if (warp == 0) {
      int carry = 0;
      for (int base = 0; base < T; base += 32) {
        const int idx = base + lane;
        int v = idx < T ? pref[idx + 1] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int n = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += n;
        }
        if (idx < T) pref[idx + 1] = v + carry;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
    }
    __syncthreads();
    P = pref[T];
    G = p.grid < P ? static_cast<int64_t>(p.grid) : P;
    // tail stealing needs at least 16 pages per CTA (so that both units of a CTA are non-empty) and
    // room for 2 G + T - 1 partial slots; the same decision in every CTA
    steal_on = STEAL && !CONTIG && p.steal != nullptr && P >= 16 * G && 2 * G + T - 1 <= p.slots_cap;
    if (static_cast<int64_t>(blockIdx.x) >= G) {
      if (blockIdx.x == 0) {  // no pages at all: every row's slot range is empty
        griddep_wait();
        for (int t = tid; t < T; t += blockDim.x) p.meta[t] = make_int2(0, 0);
      }
      return;
    }
    p0 = stream_start(blockIdx.x, P, G);
    p1 = stream_start(blockIdx.x + 1, P, G);
    int lo = 0, hi = T;  // largest r with pref[r] <= p0
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pref[mid] <= p0) lo = mid; else hi = mid;
    }
    row0 = lo;
  } else {
    row0 = blockIdx.x;
    const int c = CONTIG ? p.contig_n : max(p.ctx[row0], 0);
    p0 = 0;
    p1 = (c + PG - 1) / PG;
    if (p1 == 0) {  // empty row: its slot says so
      if (tid < p.H && row0 < p.slots_cap) p.ws_lse[static_cast<int64_t>(row0) * p.H + tid] = -INFINITY;
      return;
    }
  }

  if (tid == 0) {
    misc[0] = 0;
    misc[1] = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
      mbar_init(&mready[s], 1);
    }
    fence_barrier_init();
    fence_proxy_async();
  }
  __syncthreads();

  // Walk of (row, local page) over the global page range [p0, p1); identical in every role.
  auto row_pages_base = [&](int r, int& base, int& n) {
    if (p.stream_mode) {
      base = pref[r];
      n = pref[r + 1] - pref[r];
    } else {
      base = 0;
      n = static_cast<int>(p1);
    }
  };
  // Work units of the stream mode.  Without stealing, unit c is CTA c's page range.  With it, CTA c's
  // range [s0, s1) is cut into its main unit 2c, [s0, s1 - (s1 - s0) / 8), which CTA c streams, and its
  // tail unit 2c + 1, the last eighth, which any CTA that has finished its main unit may take from the
  // shared pool.  A row's partial from unit u goes to slot u + row, whichever CTA ran the unit.
  auto cta_mid = [&](int64_t c) {
    const int64_t s0 = stream_start(c, P, G), s1 = stream_start(c + 1, P, G);
    return s1 - (s1 - s0) / 8;
  };
  auto unit_start = [&](int64_t u) -> int64_t {
    if (!steal_on) return stream_start(u, P, G);
    return (u & 1) ? cta_mid(u >> 1) : stream_start(u >> 1, P, G);
  };
  auto unit_owner = [&](int64_t pg) -> int64_t {
    const int64_t c = stream_owner(pg, P, G);
    if (!steal_on) return c;
    return 2 * c + (pg >= cta_mid(c) ? 1 : 0);
  };

  if (warp == NC) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmap);
      // pages are read once: evict them from L2 first, so that what the step reads again - the partials,
      // the combine's up-projection and window rows - stays resident
      const uint64_t stream_policy = l2_policy_evict_first();
      if constexpr (CONTIG || !STEAL) {
        // this CTA's own page range, walked the same way by the consumers
        int r = row0, base, n;
        row_pages_base(r, base, n);
        int it = 0;
        for (int64_t g = p0; g < p1; ++g, ++it) {
          while (g >= base + n) {
            ++r;
            row_pages_base(r, base, n);
          }
          const int lp = static_cast<int>(g - base);
          const int s = it % STAGES;
          if (it >= STAGES) {
            if (!mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, p.wait_ns)) {
              record_error(p.err, kErrWaitEmpty);
              atomicExch(&misc[0], 1);
              break;
            }
          }
          mbar_arrive_expect_tx(&full[s], C::PAGE_BYTES);
          if constexpr (CONTIG) {
            // keys [lp * PG, lp * PG + PG) of row r; keys past N arrive zero-filled
            tma_load_4d(stages + s * C::PAGE_BYTES, &tmap, &full[s], 0, lp * PG, 0, r);
            tma_load_4d(stages + s * C::PAGE_BYTES + (W / 64) * C::SLAB_BYTES, &tmap_v, &full[s], 0, lp * PG, 0, r);
          } else {
            const int blk = lp < p.max_blocks ? p.block_table[static_cast<int64_t>(r) * p.bt_st + lp] : -1;
            // a page outside the table or the cache loads as zeros (TMA out-of-range fill): never a read
            // outside the buffers, but the caller learns of it through the error word
            if (blk < 0 || blk >= p.num_blocks) record_error(p.err, kErrBlock);
            tma_load_4d_hint(stages + s * C::PAGE_BYTES, &tmap, &full[s], 0, 0, 0, blk, stream_policy);
          }
        }
      } else {
        // tail stealing: units of pages, each page announced to the consumers by its stage descriptor
        int it = 0;
        bool aborted = false;
        int64_t unit = p.stream_mode ? (steal_on ? 2 * static_cast<int64_t>(blockIdx.x) : blockIdx.x) : 0;
        for (;;) {
          int64_t u0 = 0, u1 = p1;
          int r = row0;
          if (p.stream_mode) {
            u0 = unit_start(unit);
            u1 = unit_start(unit + 1);
            int lo = 0, hi = T;  // the row holding page u0: largest r with pref[r] <= u0
            while (hi - lo > 1) {
              const int mid = (lo + hi) >> 1;
              if (pref[mid] <= u0) lo = mid; else hi = mid;
            }
            r = lo;
          }
          int base, n;
          row_pages_base(r, base, n);
          for (int64_t g = u0; g < u1; ++g, ++it) {
            while (g >= base + n) {
              ++r;
              row_pages_base(r, base, n);
            }
            const int lp = static_cast<int>(g - base);
            const int st = it % STAGES;
            if (it >= STAGES && !mbar_wait(&empty[st], ((it / STAGES) - 1) & 1, p.wait_ns)) {
              record_error(p.err, kErrWaitEmpty);
              atomicExch(&misc[0], 1);
              aborted = true;
              break;
            }
            const int flags = ((g == u0 || lp == 0) ? 1 : 0) | ((g + 1 == u1 || lp + 1 == n) ? 2 : 0);
            smeta[st] = make_int4(r, lp, p.stream_mode ? static_cast<int>(unit) + r : r, flags);
            mbar_arrive(&mready[st]);
            mbar_arrive_expect_tx(&full[st], C::PAGE_BYTES);
            const int blk = lp < p.max_blocks ? p.block_table[static_cast<int64_t>(r) * p.bt_st + lp] : -1;
            // a page outside the table or the cache loads as zeros (TMA out-of-range fill): never a read
            // outside the buffers, but the caller learns of it through the error word
            if (blk < 0 || blk >= p.num_blocks) record_error(p.err, kErrBlock);
            tma_load_4d_hint(stages + st * C::PAGE_BYTES, &tmap, &full[st], 0, 0, 0, blk, stream_policy);
          }
          if (aborted || !steal_on) break;
          const unsigned ticket = atomicAdd(&p.steal[0], 1u);
          if (ticket >= static_cast<unsigned>(G)) break;
          unit = 2 * static_cast<int64_t>(ticket) + 1;
        }
        if (!aborted) {
          // end of this CTA's work: a descriptor without a page, completing the stage's phase
          const int st = it % STAGES;
          if (it < STAGES || mbar_wait(&empty[st], ((it / STAGES) - 1) & 1, p.wait_ns)) {
            smeta[st] = make_int4(-1, 0, 0, 0);
            mbar_arrive(&mready[st]);
            mbar_arrive(&full[st]);
          } else {
            record_error(p.err, kErrWaitEmpty);
          }
        }
        // the last CTA out re-zeroes the pool for the next launch (every CTA has drawn its last ticket)
        if (steal_on && atomicAdd(&p.steal[1], 1u) == static_cast<unsigned>(G) - 1) {
          atomicExch(&p.steal[0], 0u);
          atomicExch(&p.steal[1], 0u);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // Launched as a programmatic dependent of the launch that writes q (HistoryArgs::pdl), this grid
  // has been streaming pages meanwhile; q is read only after that launch has completed.  Only then
  // may this grid's own dependent (the fused combine, which also reads that launch's outputs before
  // its own wait) start on the SMs this grid frees.  Both are no-ops for an ordinary launch.
  griddep_wait();
  if (tid == 0) griddep_launch_dependents();
  if (p.stream_mode && blockIdx.x == 0) {
    // each row's slot range, written only after the wait: until the launch this grid waited for has
    // completed, a combine before it may still be reading the workspace
    for (int t = tid; t < T; t += NC * 32) {
      const int a = pref[t], b = pref[t + 1];
      int2 m = make_int2(0, 0);
      if (b > a) {
        const int lo = static_cast<int>(unit_owner(a)) + t;
        const int hi = static_cast<int>(unit_owner(b - 1)) + t + 1;
        m = make_int2(lo, hi);
      }
      p.meta[t] = m;
    }
  }
  const int g8 = lane >> 2, c4 = lane & 3;
  const int col0 = warp * 128;  // first latent column owned by this warp
  uint32_t qa[8][4];
  float o[16][4];
  float m_run[2], l_run[2];
  int buf = 0;

  int r = row0, base, n;
  row_pages_base(r, base, n);
  int it = 0;
  bool seg_open = false;
  int ctx_r = 0;

  for (int64_t g = p0;; ++g, ++it) {
    const int s = it % STAGES;
    int lp = 0, slot = 0;
    bool seg_start, seg_end, stop = false;
    if constexpr (CONTIG || !STEAL) {
      if (g >= p1) break;  // the same in every consumer warp
      while (g >= base + n) {
        ++r;
        row_pages_base(r, base, n);
      }
      lp = static_cast<int>(g - base);
      seg_start = !seg_open;
      seg_end = (g + 1 == p1) || (lp + 1 == n);
      slot = p.stream_mode ? static_cast<int>(blockIdx.x) + r : r;
    } else {
      // the page's descriptor (its row, local page, partial slot and segment flags) or the end mark
      const bool ok_m = mbar_wait(&mready[s], (it / STAGES) & 1, p.wait_ns);
      const int4 m = ok_m ? smeta[s] : make_int4(-1, 0, 0, 0);
      if (!ok_m) {
        record_error(p.err, kErrWaitFull);
        misc[1] = 1;
      }
      stop = m.x < 0;
      if (!stop) r = m.x;
      lp = m.y;
      slot = m.z;
      seg_start = !stop && (m.w & 1);
      seg_end = !stop && (m.w & 2);
    }
    if (seg_start) {
      seg_open = true;
      ctx_r = CONTIG ? p.contig_n : max(p.ctx[r], 0);
      const __nv_bfloat16* qr = p.q + static_cast<int64_t>(r) * p.q_st;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int d = col0 + kk * 16 + 2 * c4;
        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(qr + static_cast<int64_t>(g8) * p.q_sh + d);
        const uint32_t* q1 = reinterpret_cast<const uint32_t*>(qr + static_cast<int64_t>(g8 + 8) * p.q_sh + d);
        const bool h0 = g8 < p.H, h1 = g8 + 8 < p.H;
        // plain (L1-cached) loads, not the read-only path: q may have been written during this grid's
        // lifetime, by the launch griddep_wait waited for (L2-only loads measured 3% slower here)
        qa[kk][0] = h0 ? *q0 : 0u;
        qa[kk][1] = h1 ? *q1 : 0u;
        qa[kk][2] = h0 ? q0[4] : 0u;
        qa[kk][3] = h1 ? q1[4] : 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
      m_run[0] = m_run[1] = -INFINITY;
      l_run[0] = l_run[1] = 0.f;
    }
    // contiguous mode: visibility of this thread's score keys (j * 8 + 2 c4 + e), fetched before the
    // tile wait so the loads overlap it
    uint32_t vis = 0xffffffffu;
    if constexpr (CONTIG) {
      vis = 0;
      const int nk = min(PG, ctx_r - lp * PG);
      const uint8_t* mrow = p.mask + static_cast<int64_t>(r) * p.mask_st + static_cast<int64_t>(lp) * PG;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int k = j * 8 + 2 * c4 + e;
          if (k < nk && mrow[k]) vis |= 1u << (2 * j + e);
        }
    }
    const bool ok = mbar_wait(&full[s], (it / STAGES) & 1, p.wait_ns);
    if (!ok) {
      record_error(p.err, kErrWaitFull);
      misc[1] = 1;
    }
    const uint32_t sbase = smem_u32(stages + s * C::PAGE_BYTES);
    const int valid = stop ? 0 : min(PG, ctx_r - lp * PG);

    // ---- partial scores over this warp's 128 columns
    float sc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < NT / 2; ++kp) {
      const int key = kp * 16 + ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int slab = (col0 >> 6) + (kk >> 2);
        const int chunk = ((kk & 3) << 1) + ((lane >> 3) & 1);
        const uint32_t addr = sbase + slab * C::SLAB_BYTES + key * 128 + ((chunk ^ (key & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma_bf16_16816(sc[2 * kp], qa[kk], b0, b1);
        mma_bf16_16816(sc[2 * kp + 1], qa[kk], b2, b3);
      }
    }
    if constexpr (NC > 1) {
      float4* mine = xbuf + (buf * NC + warp) * NT * 32;
#pragma unroll
      for (int j = 0; j < NT; ++j) mine[j * 32 + lane] = make_float4(sc[j][0], sc[j][1], sc[j][2], sc[j][3]);
      named_bar_sync(1, NC * 32);
#pragma unroll
      for (int j = 0; j < NT; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int w = 0; w < NC; ++w) {
        const float4* part = xbuf + (buf * NC + w) * NT * 32;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const float4 v = part[j * 32 + lane];
          sc[j][0] += v.x; sc[j][1] += v.y; sc[j][2] += v.z; sc[j][3] += v.w;
        }
      }
      buf ^= 1;
      // uniform across consumer warps: every setter wrote misc[1] before this barrier, and every warp
      // read the same descriptor (a warp whose wait ran out took it as the end and set misc[1])
      if (misc[1] || stop) break;
    } else {
      if (misc[1] || stop) break;
    }

    // ---- online softmax (log2 domain); keys >= valid are masked
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int k0 = j * 8 + 2 * c4;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool in = CONTIG ? ((vis >> (2 * j + e)) & 1u) != 0 : (k0 + e) < valid;
        sc[j][e] = in ? sc[j][e] * p.scale_log2 : -INFINITY;
        sc[j][2 + e] = in ? sc[j][2 + e] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, sc[j][e]);
        mx1 = fmaxf(mx1, sc[j][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
    // contiguous mode: a row whose keys so far are all masked keeps max -inf; shift by 0 so it
    // contributes 0, not NaN (paged pages always hold a visible first key, so their max is finite)
    const float sf0 = (CONTIG && mn0 == -INFINITY) ? 0.f : mn0, sf1 = (CONTIG && mn1 == -INFINITY) ? 0.f : mn1;
    const float al0 = exp2f(m_run[0] - sf0), al1 = exp2f(m_run[1] - sf1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[NT / 2][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const float e0 = exp2f(sc[j][0] - sf0), e1 = exp2f(sc[j][1] - sf0);
      const float e2 = exp2f(sc[j][2] - sf1), e3 = exp2f(sc[j][3] - sf1);
      rs0 += e0 + e1;
      rs1 += e2 + e3;
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16(e0, e1);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16(e2, e3);
    }
    l_run[0] = l_run[0] * al0 + rs0;
    l_run[1] = l_run[1] * al1 + rs1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= al0; o[j][1] *= al0;
      o[j][2] *= al1; o[j][3] *= al1;
    }

    // ---- O += P . V over this warp's columns
#pragma unroll
    for (int ks = 0; ks < NT / 2; ++ks) {
      const int key = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int kb0 = ks * 16 + 2 * c4, kb1 = kb0 + 8;  // keys of (b0|b2) and (b1|b3) pairs
#pragma unroll
      for (int jd = 0; jd < 8; ++jd) {
        const int dcol = col0 + jd * 16;
        const int slab = (W >> 6) + (dcol >> 6);
        const int chunk = ((dcol & 63) >> 3) + (lane >> 4);
        const uint32_t addr = sbase + slab * C::SLAB_BYTES + key * 128 + ((chunk ^ (key & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(addr, b0, b1, b2, b3);
        if (valid < PG) {
          b0 = mask_pair(b0, kb0, valid);
          b1 = mask_pair(b1, kb1, valid);
          b2 = mask_pair(b2, kb0, valid);
          b3 = mask_pair(b3, kb1, valid);
        }
        mma_bf16_16816(o[2 * jd], pa[ks], b0, b1);
        mma_bf16_16816(o[2 * jd + 1], pa[ks], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    // ---- segment end: write the normalised partial and its lse
    if (seg_end) {
      seg_open = false;
      float l0 = l_run[0], l1 = l_run[1];
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      if (slot >= p.slots_cap) {
        record_error(p.err, kErrSlots);
      } else {
        float inv0 = 1.f / l0, inv1 = 1.f / l1;
        if constexpr (CONTIG) {  // a segment with every key masked: o = 0, lse = -inf
          if (!(l0 > 0.f)) inv0 = 0.f;
          if (!(l1 > 0.f)) inv1 = 0.f;
        }
        float* base0 = p.ws_o + (static_cast<int64_t>(slot) * p.H + g8) * W;
        float* base1 = p.ws_o + (static_cast<int64_t>(slot) * p.H + g8 + 8) * W;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int d = col0 + j * 8 + 2 * c4;
          if (g8 < p.H) *reinterpret_cast<float2*>(base0 + d) = make_float2(o[j][0] * inv0, o[j][1] * inv0);
          if (g8 + 8 < p.H) *reinterpret_cast<float2*>(base1 + d) = make_float2(o[j][2] * inv1, o[j][3] * inv1);
        }
        if (warp == 0 && c4 == 0) {
          const float ln2 = 0.6931471805599453f;
          if (g8 < p.H) p.ws_lse[static_cast<int64_t>(slot) * p.H + g8] = (m_run[0] + log2f(l0)) * ln2;
          if (g8 + 8 < p.H) p.ws_lse[static_cast<int64_t>(slot) * p.H + g8 + 8] = (m_run[1] + log2f(l1)) * ln2;
        }
      }
    }
  }
}

// Stage-2 reduce: partials of row t -> o[t, h, :] (bf16 and/or fp32) and lse[h, t].
// Stage-2 merge of one (row t, head h), 128 columns (chunk blockIdx.z) per CTA: the LSE-weighted
// mean of the row's split partials (slots [lo, hi) from meta in stream mode, else slot t) and its
// lse.  A long row can have ~100 partials (a few rows over a whole GPU), so the slots are spread
// over kReduceLanes slot-lanes (one warp each; 32 threads = 32 float4 columns): a warp loads the lse
// and the column values of up to kReduceU of its slots in ONE memory round, the CTA agrees on the
// running max through shared memory, and each thread accumulates its column; more slots take more
// passes with an online rescale.  The lanes are summed through shared memory.  Thread (lane 0, c)
// returns columns 128 z + 4c .. + 3 (other lanes return zeros).  An empty row (flagged, or no partial
// with a finite lse) gives 0 and -inf.
constexpr int kReduceLanes = 8, kReduceCols = 32, kReduceThreads = kReduceLanes * kReduceCols;
constexpr int kReduceU = 12;  // slots per slot-lane in one pass: 96 slots per pass

template <int W>
__device__ __forceinline__ float4 reduce_row(const float* __restrict__ ws_o, const float* __restrict__ ws_lse,
                                             const int2* __restrict__ meta, int stream_mode, int t, int h, int H,
                                             const uint8_t* __restrict__ empty, float& lse) {
  __shared__ float red[kReduceLanes];
  __shared__ float sums[kReduceLanes];
  __shared__ float4 part[(kReduceLanes - 1) * kReduceCols];
  const int tid = threadIdx.x, col = tid % kReduceCols, lane = tid / kReduceCols;  // lane = warp
  const int colg = blockIdx.z * kReduceCols + col;  // float4 column of the row
  int lo, hi;
  if (stream_mode) {
    const int2 m = meta[t];
    lo = m.x;
    hi = m.y;
  } else {
    lo = t;
    hi = t + 1;
  }
  const int n = (empty && empty[t]) ? 0 : hi - lo;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f, mx = -INFINITY;  // mx: the CTA's running max (the same in every thread)
  for (int base = 0; base < n; base += kReduceLanes * kReduceU) {
    float ls[kReduceU];
    float4 v[kReduceU];
    float pm = -INFINITY;
#pragma unroll
    for (int u = 0; u < kReduceU; ++u) {  // one round: every load of this pass in flight together
      const int i = base + lane + u * kReduceLanes;
      const int64_t slot = lo + (i < n ? i : 0);
      ls[u] = i < n ? ws_lse[slot * H + h] : -INFINITY;
      v[u] = i < n ? reinterpret_cast<const float4*>(ws_o + (slot * H + h) * W)[colg] : make_float4(0.f, 0.f, 0.f, 0.f);
      pm = fmaxf(pm, ls[u]);
    }
    if (col == 0) red[lane] = pm;
    __syncthreads();
    float m2 = mx;
#pragma unroll
    for (int l = 0; l < kReduceLanes; ++l) m2 = fmaxf(m2, red[l]);
    __syncthreads();  // red is read by every thread before the next pass writes it
    if (m2 == -INFINITY) continue;
    if (m2 != mx) {
      const float sc = expf(mx - m2);  // 0 while nothing has been summed (mx = -inf)
      wsum *= sc;
      acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
      mx = m2;
    }
#pragma unroll
    for (int u = 0; u < kReduceU; ++u) {
      if (ls[u] == -INFINITY) continue;  // past the row's slots, or a slot without keys
      const float w = expf(ls[u] - mx);
      wsum += w;
      acc.x += w * v[u].x; acc.y += w * v[u].y; acc.z += w * v[u].z; acc.w += w * v[u].w;
    }
  }
  if (lane > 0) part[(lane - 1) * kReduceCols + col] = acc;
  if (col == 0) sums[lane] = wsum;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int l = 0; l < kReduceLanes; ++l) total += sums[l];
  const bool is_empty = mx == -INFINITY;
  if (lane == 0) {
#pragma unroll
    for (int l = 1; l < kReduceLanes; ++l) {
      const float4 v = part[(l - 1) * kReduceCols + col];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (!is_empty) {
      const float inv = 1.f / total;
      acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
    } else {
      acc = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  lse = is_empty ? -INFINITY : mx + logf(total);
  return acc;
}

template <int W>
__global__ void __launch_bounds__(kReduceThreads, 1) history_reduce_kernel(const float* __restrict__ ws_o,
                                                                         const float* __restrict__ ws_lse,
                                                                         const int2* __restrict__ meta,
                                                                         int stream_mode, int T, int H,
                                                                         const uint8_t* __restrict__ empty,
                                                                         __nv_bfloat16* __restrict__ out,
                                                                         int64_t o_st, int64_t o_sh,
                                                                         float* __restrict__ out_f32,
                                                                         float* __restrict__ lse_out,
                                                                         int64_t lse_st, int64_t lse_sh) {
  // launched as a programmatic dependent of the split: it waits for the split grid before its first
  // read, and lets its own dependent (a combine, which waits for this grid before it reads z) start now
  griddep_launch_dependents();
  griddep_wait();
  const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  float lse;
  const float4 acc = reduce_row<W>(ws_o, ws_lse, meta, stream_mode, t, h, H, empty, lse);
  if (tid >= kReduceCols) return;
  const int c = (blockIdx.z * kReduceCols + tid) * 4;
  if (out) {
    __nv_bfloat16* dst = out + static_cast<int64_t>(t) * o_st + static_cast<int64_t>(h) * o_sh + c;
    reinterpret_cast<__nv_bfloat162*>(dst)[0] = __floats2bfloat162_rn(acc.x, acc.y);
    reinterpret_cast<__nv_bfloat162*>(dst)[1] = __floats2bfloat162_rn(acc.z, acc.w);
  }
  if (out_f32) *reinterpret_cast<float4*>(out_f32 + (static_cast<int64_t>(t) * H + h) * W + c) = acc;
  if (tid == 0 && blockIdx.z == 0 && lse_out) lse_out[static_cast<int64_t>(h) * lse_sh + t * lse_st] = lse;
}

// Stage-2 merge for rows with few partials (the usual decode and contiguous-reader case: about
// grid / T + 1 slots per row): one warp per (row t, head h), all W columns - lane l holds float4
// columns l, l + 32, ... - and the slots' lse and rows loaded together, up to 4 (W = 1024: 2) slots
// per memory round, with an online rescale when a later round raises the max.  Launched as a
// programmatic dependent of the split (reduce_pdl): it waits for the split grid before its first
// read.  Same outputs as history_reduce_kernel.
constexpr int kReduceWarpHeads = 4;  // warps (rows x heads) per CTA
template <int W>
__global__ void __launch_bounds__(32 * kReduceWarpHeads)
    history_reduce_warp_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse,
                               const int2* __restrict__ meta, int stream_mode, int T, int H,
                               const uint8_t* __restrict__ empty, __nv_bfloat16* __restrict__ out, int64_t o_st,
                               int64_t o_sh, float* __restrict__ out_f32, float* __restrict__ lse_out, int64_t lse_st,
                               int64_t lse_sh) {
  griddep_wait();
  constexpr int NV = W / 128, U = NV > 4 ? 2 : 4;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x * kReduceWarpHeads + (threadIdx.x >> 5);
  if (pair >= T * H) return;
  const int t = pair / H, h = pair % H;
  int lo = t, hi = t + 1;
  if (stream_mode) {
    const int2 m = meta[t];
    lo = m.x;
    hi = m.y;
  }
  float4 acc[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  float mx = -INFINITY, wsum = 0.f;
  if (!(empty && empty[t])) {
    for (int s0 = lo; s0 < hi; s0 += U) {
      float ls[U];
      float4 v[U][NV];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int s = s0 + u;
        ls[u] = s < hi ? ws_lse[static_cast<int64_t>(s) * H + h] : -INFINITY;
        const float4* src = reinterpret_cast<const float4*>(ws_o + (static_cast<int64_t>(s < hi ? s : lo) * H + h) * W);
#pragma unroll
        for (int i = 0; i < NV; ++i) v[u][i] = s < hi ? src[i * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float m2 = mx;
#pragma unroll
      for (int u = 0; u < U; ++u) m2 = fmaxf(m2, ls[u]);
      if (m2 == -INFINITY) continue;
      if (m2 != mx) {
        const float sc = expf(mx - m2);  // 0 while nothing has been summed
        wsum *= sc;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          acc[i].x *= sc; acc[i].y *= sc; acc[i].z *= sc; acc[i].w *= sc;
        }
        mx = m2;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (ls[u] == -INFINITY) continue;
        const float w = expf(ls[u] - mx);
        wsum += w;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          acc[i].x += w * v[u][i].x; acc[i].y += w * v[u][i].y; acc[i].z += w * v[u][i].z; acc[i].w += w * v[u][i].w;
        }
      }
    }
  }
  const bool is_empty = mx == -INFINITY;
  const float inv = is_empty ? 0.f : 1.f / wsum;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4 r = make_float4(acc[i].x * inv, acc[i].y * inv, acc[i].z * inv, acc[i].w * inv);
    const int c = (i * 32 + lane) * 4;
    if (out) {
      __nv_bfloat16* dst = out + static_cast<int64_t>(t) * o_st + static_cast<int64_t>(h) * o_sh + c;
      reinterpret_cast<__nv_bfloat162*>(dst)[0] = __floats2bfloat162_rn(r.x, r.y);
      reinterpret_cast<__nv_bfloat162*>(dst)[1] = __floats2bfloat162_rn(r.z, r.w);
    }
    if (out_f32) *reinterpret_cast<float4*>(out_f32 + (static_cast<int64_t>(t) * H + h) * W + c) = r;
  }
  if (lane == 0 && lse_out) lse_out[static_cast<int64_t>(h) * lse_sh + t * lse_st] = is_empty ? -INFINITY : mx + logf(wsum);
}

// The sequence-split exchange fused into the reduce: this GPU's part - z [T, H, W] followed by lse
// [H, T], as exchange words tagged epoch + 1 - is stored straight into every rank's receive slot
// (peer memory over NVLink, this GPU's own slot included).  The receivers poll the words, so the
// kernel ends with its stores: no fence, flag or CTA counter.  Launched as a programmatic dependent
// of the history kernel (griddepcontrol), it releases its own dependent - the combine - before it
// waits for the history grid: the combine's window phase, whose inputs were complete before the
// history kernel passed its own wait, then overlaps the history's tail and this reduce, and its
// merge consumes each remote row as it lands.
template <int W>
__global__ void __launch_bounds__(kReduceThreads)
    history_reduce_exchange_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse,
                                   const int2* __restrict__ meta, int stream_mode, int T, int H,
                                   const uint8_t* __restrict__ empty, const ExchangeTargets x) {
  griddep_launch_dependents();
  griddep_wait();
  const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  float lse;
  const float4 acc = reduce_row<W>(ws_o, ws_lse, meta, stream_mode, t, h, H, empty, lse);
  if (tid < kReduceCols) {
    // the slot's use counter was last advanced by the combine of its previous use, which completed
    // before this grid started (stream order)
    const uint32_t tag = static_cast<uint32_t>(*x.epoch) + 1u;
    const int64_t zoff = (static_cast<int64_t>(t) * H + h) * W + (blockIdx.z * kReduceCols + tid) * 4;
    const int64_t loff = static_cast<int64_t>(T) * H * W + static_cast<int64_t>(h) * T + t;
    const bool lse_here = tid == 0 && blockIdx.z == 0;
    const uint64_t w0 = exchange_word(acc.x, tag), w1 = exchange_word(acc.y, tag);
    const uint64_t w2 = exchange_word(acc.z, tag), w3 = exchange_word(acc.w, tag);
    const uint64_t wl = exchange_word(lse, tag);
#pragma unroll
    for (int d = 0; d < kMaxExchangeRanks; ++d) {  // constant indices keep the targets in registers
      if (d >= x.world) break;
      st_words2(x.part[d] + zoff, w0, w1);
      st_words2(x.part[d] + zoff + 2, w2, w3);
      if (lse_here) st_word(x.part[d] + loff, wl);
    }
  }
}

// ------------------------------------------------------------------ host side
template <int W, int PG>
size_t history_smem_bytes(int T) {
  using C = HistoryCfg<W, PG>;
  // stages, score exchange, full / empty / descriptor-ready barriers, stage descriptors, misc, prefix
  return 1024 + static_cast<size_t>(C::STAGES) * C::PAGE_BYTES + C::XBUF_BYTES + 3 * C::STAGES * 8 +
         16 * C::STAGES + 16 + 4 * (static_cast<size_t>(T) + 1);
}

// Pools of the split kernel's tail stealing: two counters (ticket, CTAs done) per workspace, zero
// between launches - each launch's last CTA re-zeroes its pair.  A workspace pointer keeps its pair
// for the life of the process (up to kStealSlots workspaces; later ones run without stealing).  Two
// launches on one workspace are ordered anyway (they share its partial slots), so a pair is never
// used by two kernels at once.  The array is a file-scope device variable: its address in the current
// context is looked up once per context; a look-up that would happen during a stream capture is
// skipped and that launch runs without stealing.
constexpr int kStealSlots = 1024;
static __device__ unsigned g_steal[kStealSlots][2];

static unsigned* steal_counters(const void* ws, cudaStream_t stream) {
  constexpr int kCtxSlots = 64;
  static std::mutex mu;
  static const void* keys[kStealSlots];
  static int nkeys = 0;
  static CUcontext ctxs[kCtxSlots] = {nullptr};
  static unsigned* bases[kCtxSlots] = {nullptr};
  static int nctx = 0, next_ctx = 0;
  CtxGetCurrent get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (!get || get(&ctx) != CUDA_SUCCESS || !ctx) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  unsigned* base = nullptr;
  for (int i = 0; i < nctx; ++i)
    if (ctxs[i] == ctx) base = bases[i];
  if (!base) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_steal) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    const int slot = nctx < kCtxSlots ? nctx++ : (next_ctx++ % kCtxSlots);
    ctxs[slot] = ctx;
    bases[slot] = base = static_cast<unsigned*>(ptr);
  }
  for (int i = 0; i < nkeys; ++i)
    if (keys[i] == ws) return base + 2 * i;
  if (nkeys == kStealSlots) return nullptr;
  keys[nkeys] = ws;
  return base + 2 * nkeys++;
}

// CTAs per SM of the split kernel at its largest shared-memory footprint (queried once per device).
template <int W, int PG>
static int occupancy_for() {
  using C = HistoryCfg<W, PG>;
  static unsigned attr_mask = 0;
  static int cached[32] = {0};
  const size_t smem = history_smem_bytes<W, PG>(kHistoryMaxStreamRows);
  ensure_smem_limit(history_split_kernel<W, PG>, static_cast<int>(smem), attr_mask);
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 31;
  if (cached[dev] < 1) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, history_split_kernel<W, PG>, C::THREADS, smem) !=
            cudaSuccess ||
        n < 1)
      return 1;  // no device here: do not cache the fallback
    cached[dev] = n;
  }
  return cached[dev];
}


template <int W, int PG>
static int launch_split(const HistoryArgs& a, const HistoryPlan& plan, cudaStream_t stream) {
  using C = HistoryCfg<W, PG>;
  CUtensorMap tmap;
  int rc = latent_cache_tmap(&tmap, a.cache, a.num_blocks, a.cache_st_block, a.cache_st_row, W, PG);
  if (rc) return rc;
  HistoryParams p;
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_st = a.q_st;
  p.q_sh = a.q_sh;
  p.block_table = a.block_table;
  p.bt_st = a.bt_st;
  p.max_blocks = a.max_blocks;
  p.ctx = a.ctx;
  p.T = a.T;
  p.H = a.H;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.ws_o = plan.ws_o;
  p.ws_lse = plan.ws_lse;
  p.meta = plan.meta;
  p.slots_cap = plan.slots_cap;
  p.grid = plan.grid;
  p.stream_mode = plan.stream_mode;
  p.err = a.err;
  p.wait_ns = wait_limit_ns();
  p.num_blocks = a.num_blocks;
  const size_t smem = history_smem_bytes<W, PG>(plan.stream_mode ? a.T : 0);
  occupancy_for<W, PG>();
  p.contig_n = 0;
  p.mask = nullptr;
  p.mask_st = 0;
  // tail stealing when the workspace holds 2 G + T - 1 slots (the kernel also wants 16 pages per CTA)
  // Tail stealing (the STEAL kernel) doubles a row's partials, which the combine merges in series: only
  // where rows are about as many as CTAs (at most 2 CTAs per row on average) and the workspace holds
  // 2 G + T - 1 slots.  The kernel itself also wants 16 pages per CTA, or keeps its static ranges.
  p.steal = (plan.stream_mode && plan.grid <= 2 * a.T && 2 * static_cast<int64_t>(plan.grid) + a.T - 1 <= plan.slots_cap)
                ? steal_counters(a.ws, stream) : nullptr;
  auto kernel = p.steal ? history_split_kernel<W, PG, false, true> : history_split_kernel<W, PG, false, false>;
  if (p.steal) {
    static unsigned steal_mask = 0;
    ensure_smem_limit(history_split_kernel<W, PG, false, true>,
                      static_cast<int>(history_smem_bytes<W, PG>(kHistoryMaxStreamRows)), steal_mask);
  }
  if (!a.pdl) {
    kernel<<<plan.grid, C::THREADS, smem, stream>>>(tmap, tmap, p);
    return cuda_status(cudaGetLastError(), "history_split_kernel launch");
  }
  // programmatic dependent of the preceding launch (the one that writes q): pages stream meanwhile
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, tmap, tmap, p), "history_split_kernel launch");
}

int history_plan(const HistoryArgs& a, HistoryPlan* plan) {
  // Workspace accounting mirrors s6_ops.S6Workspace.attn_logits (s6_ops.py:109-114): the op may use
  // T * splits * H * (W + 1) floats and raises when the buffer is smaller.
  const int64_t need = static_cast<int64_t>(a.T) * a.num_kv_splits * a.H * (a.W + 1);
  if (need > a.ws_floats) {
    set_error("S6 workspace overflow: need %lld floats, have %lld", static_cast<long long>(need),
              static_cast<long long>(a.ws_floats));
    return kStatusOverflow;
  }
  const int64_t per_slot = static_cast<int64_t>(a.H) * (a.W + 1);
  const int64_t meta_floats = 2 * static_cast<int64_t>(a.T);
  int sms = 148, occ = 1;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  switch (a.W * 100 + a.page) {
    case 25616: occ = occupancy_for<256, 16>(); break;
    case 25632: occ = occupancy_for<256, 32>(); break;
    case 51216: occ = occupancy_for<512, 16>(); break;
    case 51232: occ = occupancy_for<512, 32>(); break;
    case 102416: occ = occupancy_for<1024, 16>(); break;
    default: break;
  }
  const int64_t stream_slots = (need - meta_floats) / per_slot;
  const int64_t g_stream = std::min<int64_t>(static_cast<int64_t>(sms) * occ * a.waves, stream_slots - a.T + 1);
  if (a.num_kv_splits >= 2 && a.T <= kHistoryMaxStreamRows && g_stream >= 1 && a.T >= 1) {
    plan->stream_mode = 1;
    plan->grid = static_cast<int>(g_stream);
    plan->slots_cap = static_cast<int>(stream_slots);
  } else {
    plan->stream_mode = 0;
    plan->grid = a.T;
    plan->slots_cap = static_cast<int>(need / per_slot);
  }
  plan->ws_o = a.ws;
  plan->ws_lse = a.ws + static_cast<int64_t>(plan->slots_cap) * a.H * a.W;
  plan->meta = reinterpret_cast<int2*>(plan->ws_lse + static_cast<int64_t>(plan->slots_cap) * a.H);
  if (plan->stream_mode && (reinterpret_cast<uintptr_t>(plan->meta) & 7)) {
    // keep int2 alignment: shift the metadata one float up (still inside `need`)
    plan->meta = reinterpret_cast<int2*>(plan->ws_lse + static_cast<int64_t>(plan->slots_cap) * a.H + 1);
    if (static_cast<int64_t>(plan->slots_cap) * per_slot + meta_floats + 1 > need) {
      plan->slots_cap -= 1;
      plan->grid = std::min(plan->grid, plan->slots_cap - a.T + 1);
      plan->ws_lse = a.ws + static_cast<int64_t>(plan->slots_cap) * a.H * a.W;
      float* m = plan->ws_lse + static_cast<int64_t>(plan->slots_cap) * a.H;
      if (reinterpret_cast<uintptr_t>(m) & 7) ++m;
      plan->meta = reinterpret_cast<int2*>(m);
    }
  }
  return kStatusOk;
}

int history_split(const HistoryArgs& a, const HistoryPlan& plan, cudaStream_t stream) {
  if (a.T == 0) return kStatusOk;
  switch (a.W * 100 + a.page) {
    case 25616: return launch_split<256, 16>(a, plan, stream);
    case 25632: return launch_split<256, 32>(a, plan, stream);
    case 51216: return launch_split<512, 16>(a, plan, stream);
    case 51232: return launch_split<512, 32>(a, plan, stream);
    case 102416: return launch_split<1024, 16>(a, plan, stream);
    default:
      set_error("unsupported latent width %d / page %d (widths 256, 512 with pages 16, 32; width 1024 with page 16)",
                a.W, a.page);
      return kStatusInvalid;
  }
}

template <int W>
static int launch_contig(const ContigArgs& c, const HistoryPlan& plan, cudaStream_t stream) {
  constexpr int PG = 16;
  using C = HistoryCfg<W, PG>;
  CUtensorMap tk, tv;
  int rc = contig_rows_tmap(&tk, c.k, c.B, c.N, W, c.k_sb, c.k_sn, PG);
  if (rc) return rc;
  if ((rc = contig_rows_tmap(&tv, c.v, c.B, c.N, W, c.v_sb, c.v_sn, PG))) return rc;
  HistoryParams p{};
  p.q = static_cast<const __nv_bfloat16*>(c.q);
  p.q_st = c.q_sb;
  p.q_sh = c.q_sh;
  p.T = c.B;
  p.H = c.H;
  p.scale_log2 = c.scale * 1.4426950408889634f;
  p.ws_o = plan.ws_o;
  p.ws_lse = plan.ws_lse;
  p.meta = plan.meta;
  p.slots_cap = plan.slots_cap;
  p.grid = plan.grid;
  p.stream_mode = plan.stream_mode;
  p.err = c.err;
  p.wait_ns = wait_limit_ns();
  p.num_blocks = 0;
  p.contig_n = c.N;
  p.steal = nullptr;
  p.mask = c.mask;
  p.mask_st = c.m_sb;
  static unsigned attr_mask = 0;
  const size_t smem = history_smem_bytes<W, PG>(plan.stream_mode ? c.B : 0);
  ensure_smem_limit(history_split_kernel<W, PG, true>, static_cast<int>(history_smem_bytes<W, PG>(kHistoryMaxStreamRows)),
                    attr_mask);
  history_split_kernel<W, PG, true><<<plan.grid, C::THREADS, smem, stream>>>(tk, tv, p);
  return cuda_status(cudaGetLastError(), "history_split_kernel (contiguous) launch");
}

int history_attention_contig(const ContigArgs& c, cudaStream_t stream) {
  if (c.B == 0) return kStatusOk;
  HistoryArgs a{};
  a.T = c.B;
  a.H = c.H;
  a.W = c.W;
  a.page = 16;
  a.num_kv_splits = c.splits;
  a.ws = c.ws;
  a.ws_floats = c.ws_floats;
  a.waves = 1;
  a.err = c.err;
  HistoryPlan plan;
  int rc = history_plan(a, &plan);
  if (rc) return rc;
  switch (c.W) {
    case 256: rc = launch_contig<256>(c, plan, stream); break;
    case 512: rc = launch_contig<512>(c, plan, stream); break;
    case 1024: rc = launch_contig<1024>(c, plan, stream); break;
    default: set_error("contiguous history width %d unsupported (256, 512, 1024)", c.W); return kStatusInvalid;
  }
  if (rc) return rc;
  // z [B, H, W] (bf16, strided), z32 fp32 [B, H, W] contiguous, lse [B, H]
  return history_reduce_strided(a, plan, nullptr, c.z, c.z_sb, c.z_sh, c.z32, c.lse, c.H, 1, stream);
}

int history_reduce(const HistoryArgs& a, const HistoryPlan& plan, const uint8_t* empty, void* out, int64_t o_st,
                   int64_t o_sh, float* out_f32, float* lse, cudaStream_t stream) {
  return history_reduce_strided(a, plan, empty, out, o_st, o_sh, out_f32, lse, 1, a.T, stream);
}

int history_reduce_strided(const HistoryArgs& a, const HistoryPlan& plan, const uint8_t* empty, void* out,
                           int64_t o_st, int64_t o_sh, float* out_f32, float* lse, int64_t lse_st, int64_t lse_sh,
                           cudaStream_t stream) {
  if (a.T == 0) return kStatusOk;
  if (a.W != 256 && a.W != 512 && a.W != 1024) {
    set_error("unsupported latent width %d", a.W);
    return kStatusInvalid;
  }
  if (plan.stream_mode && plan.grid <= 8 * static_cast<int64_t>(a.T)) {
    // few partials per row (about grid / T + 1): warp per (row, head), launched as a programmatic
    // dependent of the split
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((static_cast<int64_t>(a.T) * a.H + kReduceWarpHeads - 1) / kReduceWarpHeads));
    cfg.blockDim = dim3(32 * kReduceWarpHeads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
    cudaError_t e;
    switch (a.W) {
      case 256: e = cudaLaunchKernelEx(&cfg, history_reduce_warp_kernel<256>, plan.ws_o, plan.ws_lse, plan.meta,
                                       plan.stream_mode, a.T, a.H, empty, o, o_st, o_sh, out_f32, lse, lse_st, lse_sh);
        break;
      case 512: e = cudaLaunchKernelEx(&cfg, history_reduce_warp_kernel<512>, plan.ws_o, plan.ws_lse, plan.meta,
                                       plan.stream_mode, a.T, a.H, empty, o, o_st, o_sh, out_f32, lse, lse_st, lse_sh);
        break;
      default: e = cudaLaunchKernelEx(&cfg, history_reduce_warp_kernel<1024>, plan.ws_o, plan.ws_lse, plan.meta,
                                      plan.stream_mode, a.T, a.H, empty, o, o_st, o_sh, out_f32, lse, lse_st, lse_sh);
        break;
    }
    return cuda_status(e, "history_reduce_warp_kernel launch");
  }
  // many partials per row (a few rows over the whole GPU): block-cooperative, also a programmatic
  // dependent of the split
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.T, a.H, a.W / (4 * kReduceCols));
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  cudaError_t e;
  switch (a.W) {
    case 256: e = cudaLaunchKernelEx(&cfg, history_reduce_kernel<256>, plan.ws_o, plan.ws_lse, plan.meta,
                                     plan.stream_mode, a.T, a.H, empty, o, o_st, o_sh, out_f32, lse, lse_st, lse_sh);
      break;
    case 512: e = cudaLaunchKernelEx(&cfg, history_reduce_kernel<512>, plan.ws_o, plan.ws_lse, plan.meta,
                                     plan.stream_mode, a.T, a.H, empty, o, o_st, o_sh, out_f32, lse, lse_st, lse_sh);
      break;
    default: e = cudaLaunchKernelEx(&cfg, history_reduce_kernel<1024>, plan.ws_o, plan.ws_lse, plan.meta,
                                    plan.stream_mode, a.T, a.H, empty, o, o_st, o_sh, out_f32, lse, lse_st, lse_sh);
      break;
  }
  return cuda_status(e, "history_reduce_kernel launch");
}

int history_reduce_exchange(const HistoryArgs& a, const HistoryPlan& plan, const uint8_t* empty,
                            const ExchangeTargets& x, bool pdl, cudaStream_t stream) {
  if (a.T == 0) return kStatusOk;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.T, a.H, a.W / (4 * kReduceCols));
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e;
  switch (a.W) {
    case 256: e = cudaLaunchKernelEx(&cfg, history_reduce_exchange_kernel<256>, plan.ws_o, plan.ws_lse,
                                     static_cast<const int2*>(plan.meta), plan.stream_mode, a.T, a.H, empty, x);
      break;
    case 512: e = cudaLaunchKernelEx(&cfg, history_reduce_exchange_kernel<512>, plan.ws_o, plan.ws_lse,
                                     static_cast<const int2*>(plan.meta), plan.stream_mode, a.T, a.H, empty, x);
      break;
    case 1024: e = cudaLaunchKernelEx(&cfg, history_reduce_exchange_kernel<1024>, plan.ws_o, plan.ws_lse,
                                      static_cast<const int2*>(plan.meta), plan.stream_mode, a.T, a.H, empty, x);
      break;
    default: set_error("unsupported latent width %d", a.W); return kStatusInvalid;
  }
  return cuda_status(e, "history_reduce_exchange_kernel launch");
}

}  // namespace hla
