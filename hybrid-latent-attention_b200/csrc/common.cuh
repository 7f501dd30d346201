// Shared device helpers for the S6 sm_100a kernels: mbarriers, TMA bulk-tensor loads,
// ldmatrix / mma.sync fragments, bf16 packing and bounded waits.
//
// Every wait on an mbarrier or a peer's exchange words is bounded by a limit in nanoseconds of device time
// (%globaltimer) that the launch passes in its parameters (hla_s6_set_wait_limit_ns, default
// kDefaultWaitNs); when it runs out the kernel records an error code in the caller's error word
// and the caller's loops unwind, so a lost copy turns into a status, never into a hung GPU.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hla {

constexpr uint64_t kDefaultWaitNs = 2000000000ull;  // 2 s of device time before a wait gives up

// Error codes written to the optional device error word (first writer wins).
enum : int {
  kErrNone = 0,
  kErrWaitFull = 1,    // consumer gave up waiting for a page copy
  kErrWaitEmpty = 2,   // producer gave up waiting for a free stage
  kErrSlots = 3,       // a partial would land outside the workspace
  kErrWaitPeer = 4,    // gave up waiting for another GPU's part of a sequence-split exchange
  kErrBlock = 5,       // a block-table entry outside the cache (the page reads as zeros)
};

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- exchange words (peer memory)
// A sequence-split part travels as 8-byte words: an fp32 value in the low half and the tag of the
// exchange it belongs to in the high half.  An aligned 8-byte access is single-copy atomic, so a
// reader that sees the expected tag in a word sees that word's value: the receiver polls the
// words themselves and no fence or flag stands between the sender's stores and their use.  The
// 16-byte accesses below are two such words each (each checked on its own).  Volatile global
// accesses are relaxed at system scope: they bypass the non-coherent L1 and see NVLink stores.
__device__ __forceinline__ uint64_t exchange_word(float v, uint32_t tag) {
  return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_words2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void st_word(uint64_t* p, uint64_t a) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ void ld_words2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t a;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}
__device__ __forceinline__ bool word_tagged(uint64_t w, uint32_t tag) { return static_cast<uint32_t>(w >> 32) == tag; }
__device__ __forceinline__ float word_value(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }

// Bounded poll of exchange words for one thread: `limit_ns` of device time counted from the first
// word that was not there yet, over all the thread's words.  The words passed in are the ones
// already loaded; after a timeout a word that is there is still taken, one that is not is reported
// missing at once (the caller records the error and uses zeros).
struct WordPoll {
  uint32_t tag;
  uint64_t limit_ns;
  uint64_t t0 = 0;
  bool failed = false;
  __device__ WordPoll(uint32_t tag_, uint64_t limit) : tag(tag_), limit_ns(limit) {}
  // false when the words are still missing once the limit has run out
  __device__ __forceinline__ bool wait2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    for (uint32_t it = 0; !(word_tagged(a, tag) && word_tagged(b, tag)); ++it) {
      if (failed) return false;
      if (t0 == 0) t0 = global_ns();
      else if ((it & 15u) == 15u && global_ns() - t0 > limit_ns) failed = true;
      ld_words2(p, a, b);
    }
    return true;
  }
  __device__ __forceinline__ bool wait1(const uint64_t* p, uint64_t& a) {
    for (uint32_t it = 0; !word_tagged(a, tag); ++it) {
      if (failed) return false;
      if (t0 == 0) t0 = global_ns();
      else if ((it & 15u) == 15u && global_ns() - t0 > limit_ns) failed = true;
      a = ld_word(p);
    }
    return true;
  }
};

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase completed, false when `limit_ns` elapsed first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && global_ns() - t0 > limit_ns) return false;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 4-D tiled bulk-tensor load into this CTA's shared memory, completion counted on `bar`.
// No multicast: every CTA fetches its own pages.
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// tma_load_4d with an L2 cache-policy hint (createpolicy below), no multicast.
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2,
                                                 int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

// L2 policy for data read once and then dead (a streamed cache page): evicted before other lines.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bring `bytes` (a multiple of 16, 16-byte aligned address) of global memory into L2 without waiting.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 5-D form of tma_load_4d (no multicast).
__device__ __forceinline__ void tma_load_5d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// ---------------------------------------------------------------- cp.async (16-byte, L2-cached)
// src_bytes < 16 zero-fills the rest of the 16-byte destination (0 = pure zero fill, no read).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes = 16) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a shared tile whose rows are `row_bytes`
// long (a multiple of 128): chunks are XOR-swizzled by row % 8 so that ldmatrix over 8 rows of
// the same logical chunk touches 8 distinct bank groups.
__device__ __forceinline__ uint32_t swz(int row, int chunk, int row_bytes) {
  return static_cast<uint32_t>(row * row_bytes + ((chunk ^ (row & 7)) << 4));
}

// ---------------------------------------------------------------- stream-K partition
// G CTAs split P work units (pages) evenly: CTA c takes [stream_start(c), stream_start(c + 1)).
__host__ __device__ inline int64_t stream_start(int64_t c, int64_t P, int64_t G) { return c * P / G; }

// Largest CTA index c with stream_start(c) <= p.
__host__ __device__ inline int64_t stream_owner(int64_t p, int64_t P, int64_t G) {
  return ((p + 1) * G - 1) / P;
}

// ---------------------------------------------------------------- programmatic dependent launch
// wait: block until the preceding grid (launched before this one with programmatic stream
// serialization) has completed and its memory is visible; a no-op for ordinary launches.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// launch_dependents: this CTA no longer holds back the launch of the dependent grid.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- named barriers
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- ldmatrix / mma
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace hla
