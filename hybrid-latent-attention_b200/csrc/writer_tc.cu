// Prefill-size writer on the 5th-generation tensor cores (tcgen05): the same operation as
// writer_kernel in gemm_ops.cu - reg_out = bf16(reg_in + bf16(h . E^T)), optionally committed to
// the latent cache with the K half latent-RoPE'd (register.py:45-79, s6_layer.py:124-147,
// ouro_latent.py:127-129) - for many tokens (config 3: 8 x 4096 prompt tokens per loop), where the
// GEMM (M = tokens, N = 1024 or 512, K = hidden) is tensor-bound.
//
// One persistent CTA per SM walks 128 x 256 output tiles:
//   warp 0      TMA producer (h tile 128 x 64, two 128 x 64 boxes of E per stage, SWIZZLE_128B, a
//               4-stage ring that runs across tiles), and owner of the TMEM allocation (2 x 256 fp32
//               columns: two accumulators, so one tile's epilogue overlaps the next tile's MMAs)
//   warp 1      a single thread issues tcgen05.mma (M = 128, N = 256, K = 16, bf16 -> fp32, both
//               operands K-major from shared memory) and commits each stage back to the producer
//   warps 2-5   epilogue: tcgen05.ld of its 32 TMEM lanes (= tile rows), bf16 rounding, the bf16
//               register add, then the register store and/or the committed-row scatter, with
//               16-byte vector accesses.
// For a commit tile the two E boxes are rows [128j, 128j + 128) and [w/2 + 128j, ...), so the
// accumulator columns c and c + 128 are a neox RoPE pair held by the same thread.
// All mbarrier waits are bounded; a timeout records an error code and the CTA unwinds.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "decode_ops.cuh"
#include "gemm_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

constexpr int kTcM = 128, kTcN = 256, kTcK = 64, kTcStages = 4;
constexpr int kTcABytes = kTcM * kTcK * 2;                 // 16 KB
constexpr int kTcBBytes = kTcN * kTcK * 2;                 // 32 KB
constexpr int kTcStageBytes = kTcABytes + kTcBBytes;       // 48 KB
constexpr int kTcSmem = 1024 + kTcStages * kTcStageBytes + 256;
constexpr int kTcThreads = 192;

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  // K-major, SWIZZLE_128B canonical layout: rows of 128 B, 8-row groups 1024 B apart (SBO),
  // LBO unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B).
  return static_cast<uint64_t>((smem_addr & 0x3FFFF) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// bf16 x bf16 -> fp32, K-major A and B, M = 128, N = 256.
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kTcN >> 3) << 17) |
                              (uint32_t(kTcM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kTcIdesc), "r"(accumulate));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 16 consecutive fp32 TMEM columns of this thread's lane (no wait; see tmem_wait_ld).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct TcParams {
  WriterParams w;
  int n_tiles, m_tiles;
  bool v32;  // every epilogue row segment is 32-byte aligned: 256-bit accesses (else 2 x 128-bit)
};

// 32 contiguous bytes of global memory: one 256-bit access when `v32` (the address is 32-byte
// aligned), else two 128-bit ones.  A 256-bit access fills a whole L2 sector per lane and halves
// the epilogue's load / store instructions (each lane of a warp addresses its own row).
__device__ __forceinline__ void ld32(const void* p, uint4& a, uint4& b, bool v32) {
  if (v32) {
    asm volatile("ld.global.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
                 : "l"(p));
  } else {
    a = reinterpret_cast<const uint4*>(p)[0];
    b = reinterpret_cast<const uint4*>(p)[1];
  }
}
__device__ __forceinline__ void st32(void* p, const uint4& a, const uint4& b, bool v32) {
  if (v32) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(a.x), "r"(a.y), "r"(a.z),
                 "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                 : "memory");
  } else {
    reinterpret_cast<uint4*>(p)[0] = a;
    reinterpret_cast<uint4*>(p)[1] = b;
  }
}

// E rows of the two 128-row boxes of column tile j.
__device__ __forceinline__ void tc_tile_rows(const WriterParams& p, int j, int& n_lo, int& n_hi) {
  if (p.commit && j < p.w / 256) {
    n_lo = 128 * j;
    n_hi = p.w / 2 + 128 * j;
  } else if (p.commit) {
    n_lo = p.w + 256 * (j - p.w / 256);
    n_hi = n_lo + 128;
  } else {
    n_lo = 256 * j;
    n_hi = n_lo + 128;
  }
}

// Everything a thread's row of a tile needs besides the accumulator, fetched before the accumulator
// is ready so that the loads' latency hides under the tile's MMAs: the running register's values (both
// 128-column halves), the committed row's address (the slot lookup is a chain of dependent loads),
// and the first half of the RoPE cos / sin for a pair tile (the second half is loaded mid-tile).
struct TileIn {
  uint4 lo[16], hi[16];   // reg_in
  uint4 cs[4], sn[4];     // cos / sin of 32 pairs (the table half in flight)
  const __nv_bfloat16* tab;
  __nv_bfloat16* dst;
  __nv_bfloat16* rout;
};

__device__ __forceinline__ void tc_load_rope(const TileIn& in, int col, uint4* cs, uint4* sn, int half_w, bool v32) {
#pragma unroll
  for (int i = 0; i < 4; i += 2) {
    ld32(in.tab + col + 8 * i, cs[i], cs[i + 1], v32);
    ld32(in.tab + half_w + col + 8 * i, sn[i], sn[i + 1], v32);
  }
}

__device__ __forceinline__ void tc_tile_prefetch(const WriterParams& p, int t, bool live, bool pair_tile, int n_lo,
                                                 int n_hi, TileIn& in, bool v32) {
  in.tab = nullptr;
  in.dst = nullptr;
  in.rout = (p.reg_out && live) ? p.reg_out + static_cast<int64_t>(t) * p.ro_st : nullptr;
  if (!live) return;
  if (p.reg_in) {
    const __nv_bfloat16* a = p.reg_in + static_cast<int64_t>(t) * p.ri_st + n_lo;
    const __nv_bfloat16* b = p.reg_in + static_cast<int64_t>(t) * p.ri_st + n_hi;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      ld32(a + 8 * i, in.lo[i], in.lo[i + 1], v32);
      ld32(b + 8 * i, in.hi[i], in.hi[i + 1], v32);
    }
  }
  if (p.commit) {
    const int64_t pos = p.positions[t];
    const int64_t slot = token_slot(p.qsl, p.R, t, pos, p.bt, p.bt_st, p.max_blocks, p.page, p.num_blocks);
    if (slot >= 0) in.dst = p.cache + (slot / p.page) * p.c_sb + (slot % p.page) * p.c_sr;
    in.tab = p.table + clamp_pos(pos, p.max_pos) * p.tab_st;
    if (pair_tile && in.dst) tc_load_rope(in, n_lo, in.cs, in.sn, p.w / 2, v32);
  }
}

// Epilogue of one 128 x 256 tile for this thread's row: 16 + 16 columns (c0 of both halves) at a time,
// in packed bf16x2 arithmetic (the _rn forms, which are never contracted into an fma).  Each packed
// operation rounds its exact result once to bf16; on bf16
// inputs that equals the reference's fp32 operation followed by a rounding to bf16 (a product of two
// bf16 values is exact in fp32, and rounding a sum first to fp32's 24 bits and then to bf16's 8 is
// innocuous since 24 >= 2 * 8 + 2), so the values are those of the torch order bit for bit:
//   acc -> bf16,  reg = bf16(reg_in + acc),  y1 = bf16(bf16(x1 c) + bf16(-x2 s)),
//   y2 = bf16(bf16(x2 c) + bf16(x1 s)).
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ uint32_t word(const uint4& u, int i) {
  return i == 0 ? u.x : (i == 1 ? u.y : (i == 2 ? u.z : u.w));
}

__device__ __forceinline__ void tc_store_tile(const WriterParams& p, uint32_t tacc, bool live, bool pair_tile, int n_lo,
                                              int n_hi, TileIn& in, bool v32) {
#pragma unroll
  for (int c0 = 0; c0 < 128; c0 += 16) {
    uint32_t rl[16], rh[16];
    tmem_ld16(tacc + c0, rl);  // warp-collective: every lane, live or not
    tmem_ld16(tacc + 128 + c0, rh);
    tmem_wait_ld();
    if (!live) continue;
    __nv_bfloat162 lo[8], hi[8];  // columns c0 + 2i, c0 + 2i + 1 of each half
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      lo[i] = __floats2bfloat162_rn(__uint_as_float(rl[2 * i]), __uint_as_float(rl[2 * i + 1]));
      hi[i] = __floats2bfloat162_rn(__uint_as_float(rh[2 * i]), __uint_as_float(rh[2 * i + 1]));
    }
    const int clo = n_lo + c0, chi = n_hi + c0;  // global columns
    if (p.reg_in) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        lo[i] = __hadd2_rn(as_bf2(word(in.lo[c0 / 8 + i / 4], i % 4)), lo[i]);
        hi[i] = __hadd2_rn(as_bf2(word(in.hi[c0 / 8 + i / 4], i % 4)), hi[i]);
      }
    }
    uint4 olo[2], ohi[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      olo[i] = make_uint4(as_u32(lo[4 * i]), as_u32(lo[4 * i + 1]), as_u32(lo[4 * i + 2]), as_u32(lo[4 * i + 3]));
      ohi[i] = make_uint4(as_u32(hi[4 * i]), as_u32(hi[4 * i + 1]), as_u32(hi[4 * i + 2]), as_u32(hi[4 * i + 3]));
    }
    if (in.rout) {
      st32(in.rout + clo, olo[0], olo[1], v32);
      st32(in.rout + chi, ohi[0], ohi[1], v32);
    }
    if (in.dst) {
      if (pair_tile) {
        // cos / sin of pairs [c0, c0 + 16) sit in slots (c0 % 32) / 8 .. + 1 of the half in flight;
        // the next 32 pairs are fetched once this chunk has read its own
        const int q = (c0 % 32) / 8;
        const uint4 cs[2] = {in.cs[q], in.cs[q + 1]}, sn[2] = {in.sn[q], in.sn[q + 1]};
        if (c0 % 32 == 16 && c0 + 16 < 128) tc_load_rope(in, n_lo + c0 + 16, in.cs, in.sn, p.w / 2, v32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const __nv_bfloat162 c = as_bf2(word(cs[i / 4], i % 4)), sv = as_bf2(word(sn[i / 4], i % 4));
          const __nv_bfloat162 x1 = lo[i], x2 = hi[i];
          lo[i] = __hadd2_rn(__hmul2_rn(x1, c), __hneg2(__hmul2_rn(x2, sv)));
          hi[i] = __hadd2_rn(__hmul2_rn(x2, c), __hmul2_rn(x1, sv));
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          olo[i] = make_uint4(as_u32(lo[4 * i]), as_u32(lo[4 * i + 1]), as_u32(lo[4 * i + 2]), as_u32(lo[4 * i + 3]));
          ohi[i] = make_uint4(as_u32(hi[4 * i]), as_u32(hi[4 * i + 1]), as_u32(hi[4 * i + 2]), as_u32(hi[4 * i + 3]));
        }
      }
      st32(in.dst + clo, olo[0], olo[1], v32);
      st32(in.dst + chi, ohi[0], ohi[1], v32);
    }
  }
}

// Persistent: CTA b takes tiles b, b + grid, ... in (m, j) order with j fastest (the four column tiles
// of a row block run back to back and share its h tile through L2).  The smem ring runs across tile
// boundaries; TMEM holds two 256-column accumulators so the epilogue of one tile overlaps the
// main loop of the next.
__global__ void __launch_bounds__(kTcThreads, 1)
    writer_tc_kernel(const __grid_constant__ CUtensorMap tmap_h, const __grid_constant__ CUtensorMap tmap_e,
                     const TcParams tp) {
  const WriterParams& p = tp.w;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* tfull = empty + kTcStages;  // [2] accumulator ready (tcgen05.commit)
  uint64_t* tempty = tfull + 2;         // [2] accumulator drained (one arrive per epilogue warp)
  uint64_t* drained = tempty + 2;       // every issued MMA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NK = p.K / kTcK;
  const int num_tiles = tp.n_tiles * tp.m_tiles;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kTcN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmap_h);
      prefetch_tmap(&tmap_e);
      uint32_t g = 0;  // k-blocks issued so far (ring position)
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / tp.n_tiles) * kTcM, j = tile % tp.n_tiles;
        int n_lo, n_hi;
        tc_tile_rows(p, j, n_lo, n_hi);
        for (int kb = 0; kb < NK; ++kb, ++g) {
          const int s = g % kTcStages;
          if (g >= kTcStages && !mbar_wait(&empty[s], ((g / kTcStages) - 1) & 1, p.wait_ns)) {
            record_error(p.err, kErrWaitEmpty);
            ok = false;
            break;
          }
          uint8_t* a = smem + s * kTcStageBytes;
          uint8_t* b = a + kTcABytes;
          mbar_arrive_expect_tx(&full[s], kTcStageBytes);
          tma_load_2d(a, &tmap_h, &full[s], kb * kTcK, m0);
          tma_load_2d(b, &tmap_e, &full[s], kb * kTcK, n_lo);
          tma_load_2d(b + kTcBBytes / 2, &tmap_e, &full[s], kb * kTcK, n_hi);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int b = it & 1;
        if (it >= 2 && !mbar_wait(&tempty[b], ((it >> 1) - 1) & 1, p.wait_ns)) {
          record_error(p.err, kErrWaitEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + b * kTcN;
        for (int kb = 0; kb < NK; ++kb, ++g) {
          const int s = g % kTcStages;
          if (!mbar_wait(&full[s], (g / kTcStages) & 1, p.wait_ns)) {
            record_error(p.err, kErrWaitFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * kTcStageBytes), bb = a + kTcABytes;
#pragma unroll
          for (int kk = 0; kk < kTcK / 16; ++kk)
            tc_mma(d, umma_desc_sw128(a + kk * 32), umma_desc_sw128(bb + kk * 32), (kb | kk) != 0);
          tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        tc_commit(&tfull[b]);  // accumulator b complete (after a timeout: whatever was issued)
      }
      // nothing may still write TMEM when it is released
      tc_commit(drained);
      if (!mbar_wait(drained, 0, p.wait_ns)) record_error(p.err, kErrWaitFull);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. + 31 (a warp reaches only its quarter)
    const int row = quarter * 32 + lane;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int b = it & 1;
      const int m0 = (tile / tp.n_tiles) * kTcM, j = tile % tp.n_tiles;
      int n_lo, n_hi;
      tc_tile_rows(p, j, n_lo, n_hi);
      const int t = m0 + row;
      const bool pair_tile = p.commit && j < p.w / 256;
      TileIn in;
      tc_tile_prefetch(p, t, t < p.T, pair_tile, n_lo, n_hi, in, tp.v32);
      // tcgen05.ld / wait::ld are warp-collective (.sync.aligned): the wait result is made warp-uniform
      // and every lane runs the loads; rows past T only skip their global accesses
      const bool done = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (it >> 1) & 1, p.wait_ns));
      tc_fence_after();
      if (!done) {
        record_error(p.err, kErrWaitFull);
        break;
      }
      tc_store_tile(p, tmem + b * kTcN + (static_cast<uint32_t>(quarter * 32) << 16), t < p.T, pair_tile, n_lo, n_hi,
                    in, tp.v32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTcN));
  }
}

// ---------------------------------------------------------------------------------------------
// Pair version (cta_group::2): a cluster of two CTAs on two SMs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256).  CTA r of the pair stages rows [128 r, 128 r + 128)
// of the h tile and ONE of the two 128-row E boxes (r = 0: n_lo, r = 1: n_hi) - half the operand
// bytes per output that the single-CTA tile moves - and holds rows 128 r .. + 127 of the
// accumulator in its own TMEM, all 256 columns (columns 0-127 from E box n_lo, 128-255 from n_hi,
// as in the single-CTA tile).  The leader (rank 0) issues the MMAs; both CTAs' TMA loads complete
// on the leader's full barrier; the MMA commits arrive on both CTAs' empty / tfull barriers; both
// CTAs' epilogue warps release an accumulator on the leader's tempty barrier.  Each TMA load writes
// only its own CTA's shared memory.
constexpr int kT2Stages = 6;
constexpr int kT2ABytes = 128 * kTcK * 2;                  // 16 KB (this CTA's h rows)
constexpr int kT2BBytes = 128 * kTcK * 2;                  // 16 KB (this CTA's E box)
constexpr int kT2StageBytes = kT2ABytes + kT2BBytes;       // 32 KB
constexpr int kT2Smem = 1024 + kT2Stages * kT2StageBytes + 256;
// bf16 x bf16 -> fp32, K-major A and B, M = 256 (the pair), N = 256.
constexpr uint32_t kT2Idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(256 >> 3) << 17) |
                              (uint32_t(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// The shared::cluster address of a shared variable of CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t peer_smem(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}
// Arrive on an mbarrier of either CTA of the pair (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (arrivals come from the peer CTA too).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 255u && global_ns() - t0 > limit_ns) return false;
  }
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tc2_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kT2Idesc), "r"(accumulate));
}
// Arrive on the barrier at this offset in both CTAs of the pair once the MMAs issued so far complete.
__device__ __forceinline__ void tc2_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 1)
    writer_tc2_kernel(const __grid_constant__ CUtensorMap tmap_h, const __grid_constant__ CUtensorMap tmap_e,
                      const TcParams tp) {
  const WriterParams& p = tp.w;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kT2Stages * kT2StageBytes);  // leader's are used
  uint64_t* empty = full + kT2Stages;   // both CTAs
  uint64_t* tfull = empty + kT2Stages;  // [2] both CTAs
  uint64_t* tempty = tfull + 2;         // [2] leader's are used: 8 arrivals (4 epilogue warps x 2 CTAs)
  uint64_t* drained = tempty + 2;       // leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int NK = p.K / kTcK;
  const int num_tiles = tp.n_tiles * tp.m_tiles;  // m tiles of 256 rows
  const int first = static_cast<int>(cluster_id_x()), stride = static_cast<int>(cluster_count_x());

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kTcN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < kT2Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tmap(&tmap_h);
      prefetch_tmap(&tmap_e);
      uint32_t g = 0;
      bool ok = true;
      for (int tile = first; tile < num_tiles && ok; tile += stride) {
        const int m0 = (tile / tp.n_tiles) * 256 + 128 * static_cast<int>(rank), j = tile % tp.n_tiles;
        int n_lo, n_hi;
        tc_tile_rows(p, j, n_lo, n_hi);
        const int n_mine = leader ? n_lo : n_hi;
        for (int kb = 0; kb < NK; ++kb, ++g) {
          const int s = g % kT2Stages;
          if (g >= kT2Stages && !mbar_wait(&empty[s], ((g / kT2Stages) - 1) & 1, p.wait_ns)) {
            record_error(p.err, kErrWaitEmpty);
            ok = false;
            break;
          }
          uint8_t* a = smem + s * kT2StageBytes;
          // the leader's full barrier counts both CTAs' bytes
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * kT2StageBytes);
          const uint32_t bar = peer_smem(&full[s], 0);
          tma_load_2d_pair(a, &tmap_h, bar, kb * kTcK, m0);
          tma_load_2d_pair(a + kT2ABytes, &tmap_e, bar, kb * kTcK, n_mine);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (leader && lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      int it = 0;
      for (int tile = first; tile < num_tiles && ok; tile += stride, ++it) {
        const int b = it & 1;
        if (it >= 2 && !mbar_wait_cluster(&tempty[b], ((it >> 1) - 1) & 1, p.wait_ns)) {
          record_error(p.err, kErrWaitEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + b * kTcN;
        for (int kb = 0; kb < NK; ++kb, ++g) {
          const int s = g % kT2Stages;
          if (!mbar_wait(&full[s], (g / kT2Stages) & 1, p.wait_ns)) {
            record_error(p.err, kErrWaitFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * kT2StageBytes), bb = a + kT2ABytes;
#pragma unroll
          for (int kk = 0; kk < kTcK / 16; ++kk)
            tc2_mma(d, umma_desc_sw128(a + kk * 32), umma_desc_sw128(bb + kk * 32), (kb | kk) != 0);
          tc2_commit_both(&empty[s]);
        }
        tc2_commit_both(&tfull[b]);
      }
      tc2_commit_both(drained);  // the peer's copy is not waited on
      if (!mbar_wait(drained, 0, p.wait_ns)) record_error(p.err, kErrWaitFull);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5, both CTAs)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int it = 0;
    for (int tile = first; tile < num_tiles; tile += stride, ++it) {
      const int b = it & 1;
      const int m0 = (tile / tp.n_tiles) * 256 + 128 * static_cast<int>(rank), j = tile % tp.n_tiles;
      int n_lo, n_hi;
      tc_tile_rows(p, j, n_lo, n_hi);
      const int t = m0 + row;
      const bool pair_tile = p.commit && j < p.w / 256;
      TileIn in;
      tc_tile_prefetch(p, t, t < p.T, pair_tile, n_lo, n_hi, in, tp.v32);
      const bool done = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (it >> 1) & 1, p.wait_ns));
      tc_fence_after();
      if (!done) {
        record_error(p.err, kErrWaitFull);
        break;
      }
      tc_store_tile(p, tmem + b * kTcN + (static_cast<uint32_t>(quarter * 32) << 16), t < p.T, pair_tile, n_lo, n_hi,
                    in, tp.v32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(peer_smem(&tempty[b], 0));
    }
  }
  // the leader's MMAs read this CTA's shared memory and write its TMEM: neither is released before
  // both CTAs are done (the leader's MMA thread has waited for the last MMA above)
  tc_fence_before();
  cluster_sync_all();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTcN));
  }
}

// 2-D TMA map over a [rows, K] bf16 matrix with 128-row x 64-column boxes, SWIZZLE_128B.
static int rows_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride_elems) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      set_error("cuTensorMapEncodeTiled is unavailable from the driver");
      return kStatusCuda;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcK), 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for the writer operands", static_cast<int>(r));
    return kStatusCuda;
  }
  return kStatusOk;
}

// Whether writer() should use the tcgen05 path for this shape.
bool writer_tc_eligible(const WriterParams& p) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) % 16) == 0; };
  // TMA operands: 16-byte aligned bases and row strides; epilogue: 16-byte vector accesses
  return p.T >= kTcM && p.N % kTcN == 0 && p.K % kTcK == 0 && (!p.commit || p.w % 256 == 0) && a16(p.h) &&
         a16(p.E) && (p.h_st % 8) == 0 && (p.e_st % 8) == 0 && a16(p.reg_in) && (p.ri_st % 8) == 0 &&
         a16(p.reg_out) && (p.ro_st % 8) == 0 &&
         (!p.commit || (a16(p.cache) && a16(p.table) && p.c_sb % 8 == 0 && p.c_sr % 8 == 0 && p.tab_st % 8 == 0));
}

int writer_tc(const WriterParams& p, cudaStream_t s) {
  CUtensorMap th, te;
  int rc = rows_tmap(&th, p.h, p.T, p.K, p.h_st);
  if (rc) return rc;
  if ((rc = rows_tmap(&te, p.E, p.N, p.K, p.e_st))) return rc;
  static int sms[64] = {0}, pairs[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cached = dev < 64;
  if (cached && sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int nsm = cached && sms[dev] > 0 ? sms[dev] : 148;
  TcParams tp;
  tp.w = p;
  tp.w.wait_ns = wait_limit_ns();
  tp.n_tiles = p.N / kTcN;
  // 256-bit epilogue accesses need 32-byte aligned rows (column offsets are multiples of 16 elements)
  auto a32 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) % 32) == 0; };
  tp.v32 = a32(p.reg_in) && (p.ri_st % 16) == 0 && a32(p.reg_out) && (p.ro_st % 16) == 0 &&
           (!p.commit || (a32(p.cache) && a32(p.table) && p.c_sb % 16 == 0 && p.c_sr % 16 == 0 && p.tab_st % 16 == 0));
  if (p.T >= 2 * kTcM) {
    static unsigned attr2 = 0;
    ensure_smem_limit(writer_tc2_kernel, kT2Smem, attr2);
    tp.m_tiles = (p.T + 2 * kTcM - 1) / (2 * kTcM);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = kT2Smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cached && pairs[dev] == 0) {
      cfg.gridDim = dim3(nsm);
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, writer_tc2_kernel, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = nsm / 2;
      }
      pairs[dev] = n;
    }
    const int max_pairs = cached ? pairs[dev] : nsm / 2;
    const int tiles = tp.n_tiles * tp.m_tiles;
    cfg.gridDim = dim3(2 * (tiles < max_pairs ? tiles : max_pairs));
    return cuda_status(cudaLaunchKernelEx(&cfg, writer_tc2_kernel, th, te, tp), "writer_tc2_kernel launch");
  }
  static unsigned attr_mask = 0;
  ensure_smem_limit(writer_tc_kernel, kTcSmem, attr_mask);
  tp.m_tiles = (p.T + kTcM - 1) / kTcM;
  const int tiles = tp.n_tiles * tp.m_tiles;
  writer_tc_kernel<<<tiles < nsm ? tiles : nsm, kTcThreads, kTcSmem, s>>>(th, te, tp);
  return cuda_status(cudaGetLastError(), "writer_tc_kernel launch");
}

}  // namespace hla
