// C-ABI surface of libhla_s6: argument validation, error reporting, TMA descriptor cache
// and the exported history entry points.  Declarations live in include/hla_s6.h.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "../../include/hla_s6.h"
#include "hla_s6_internal.h"

namespace hla {

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

static std::atomic<uint64_t> g_wait_ns{2000000000ull};

uint64_t wait_limit_ns() { return g_wait_ns.load(std::memory_order_relaxed); }

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return kStatusOk;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return kStatusCuda;
}

// ------------------------------------------------------------------ TMA descriptors
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct TmapKey {
  const void* ptr;
  int64_t nb, sb, sr;
  int W, page, dev;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && nb == o.nb && sb == o.sb && sr == o.sr && W == o.W && page == o.page && dev == o.dev;
  }
};

static std::mutex g_tmap_mu;
static TmapKey g_tmap_keys[32];
static CUtensorMap g_tmap_vals[32];
static int g_tmap_used = 0, g_tmap_next = 0;

int latent_cache_tmap(CUtensorMap* map, const void* cache, int64_t num_blocks, int64_t st_block, int64_t st_row,
                      int W, int page) {
  if (reinterpret_cast<uintptr_t>(cache) % 16) {
    set_error("latent cache base must be 16-byte aligned");
    return kStatusInvalid;
  }
  if ((st_row * 2) % 16 || (st_block * 2) % 16 || st_row < 2 * W || st_block < 1) {
    set_error("latent cache strides must be multiples of 8 elements (row %lld, block %lld)",
              static_cast<long long>(st_row), static_cast<long long>(st_block));
    return kStatusInvalid;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  const TmapKey key{cache, num_blocks, st_block, st_row, W, page, dev};
  {
    std::lock_guard<std::mutex> lock(g_tmap_mu);
    for (int i = 0; i < g_tmap_used; ++i)
      if (g_tmap_keys[i] == key) {
        *map = g_tmap_vals[i];
        return kStatusOk;
      }
  }
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return kStatusCuda;
  }
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(page), static_cast<cuuint64_t>(2 * W / 64),
                        static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(st_row * 2), 128, static_cast<cuuint64_t>(st_block * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(page), static_cast<cuuint32_t>(2 * W / 64), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(cache), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for the latent cache", static_cast<int>(r));
    return kStatusCuda;
  }
  std::lock_guard<std::mutex> lock(g_tmap_mu);
  const int slot = g_tmap_used < 32 ? g_tmap_used++ : (g_tmap_next++ % 32);
  g_tmap_keys[slot] = key;
  g_tmap_vals[slot] = *map;
  return kStatusOk;
}

int combine_b_tmap(CUtensorMap* map, const void* B, int H, int W, int64_t b_sh, int64_t b_sk) {
  if (reinterpret_cast<uintptr_t>(B) % 16 || (b_sh * 2) % 16 || (b_sk * 2) % 16 || b_sk < 128 || H < 1) {
    set_error("decode combine: B [H, W, 128] needs a 16-byte aligned base and strides that are multiples of 8 "
              "elements (head %lld, row %lld)", static_cast<long long>(b_sh), static_cast<long long>(b_sk));
    return kStatusInvalid;
  }
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return kStatusCuda;
  }
  // (64 columns, W rows, 2 column slabs, H heads): a box of 64 rows lands as [slab][row][64]
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(W), 2, static_cast<cuuint64_t>(H)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(b_sk * 2), 128, static_cast<cuuint64_t>(b_sh * 2)};
  cuuint32_t box[4] = {64, 64, 2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(B), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for the combine's B", static_cast<int>(r));
    return kStatusCuda;
  }
  return kStatusOk;
}

int contig_rows_tmap(CUtensorMap* map, const void* base, int64_t B, int64_t N, int W, int64_t st_b, int64_t st_n,
                     int tile) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || (st_n * 2) % 16 || (st_b * 2) % 16 || st_n < W || B < 1 || N < 1) {
    set_error("contiguous K/V need a 16-byte aligned base, row strides that are multiples of 8 elements and "
              ">= width (key stride %lld, batch stride %lld)", static_cast<long long>(st_n),
              static_cast<long long>(st_b));
    return kStatusInvalid;
  }
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return kStatusCuda;
  }
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(W / 64), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(st_n * 2), 128, static_cast<cuuint64_t>(st_b * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(tile), static_cast<cuuint32_t>(W / 64), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for contiguous K/V", static_cast<int>(r));
    return kStatusCuda;
  }
  return kStatusOk;
}

// 5-D map over a per-head cache [num_blocks, kv_heads, 16, >= Lk] (LLA) starting at column 0 of `base`:
// dims (cols, 16 rows, slabs, kv head, block), slab s covering columns [s * cols, (s + 1) * cols), with
// the (2 * cols)-byte swizzle (cols = 64, 32 or 16), so a box of (cols, 16, slabs, 1, 1) lands one page
// of one KV head as [slab][row][2 * cols bytes].
struct HeadsTmapKey {
  const void* ptr;
  int64_t nb, kvh, sb_, sh, sr;
  int cols, slabs, dev;
  bool operator==(const HeadsTmapKey& o) const {
    return ptr == o.ptr && nb == o.nb && kvh == o.kvh && sb_ == o.sb_ && sh == o.sh && sr == o.sr &&
           cols == o.cols && slabs == o.slabs && dev == o.dev;
  }
};
static HeadsTmapKey g_htmap_keys[16];
static CUtensorMap g_htmap_vals[16];
static int g_htmap_used = 0, g_htmap_next = 0;

int heads_cache_tmap(CUtensorMap* map, const void* base, int64_t num_blocks, int64_t kv_heads, int64_t st_block,
                     int64_t st_head, int64_t st_row, int cols, int slabs) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || (st_row * 2) % 16 || (st_head * 2) % 16 || (st_block * 2) % 16 ||
      (cols != 64 && cols != 32 && cols != 16) || slabs < 1 || slabs > 256 || num_blocks < 1 || kv_heads < 1) {
    set_error("per-head cache: needs a 16-byte aligned base and strides that are multiples of 8 elements");
    return kStatusInvalid;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  const HeadsTmapKey key{base, num_blocks, kv_heads, st_block, st_head, st_row, cols, slabs, dev};
  {
    std::lock_guard<std::mutex> lock(g_tmap_mu);
    for (int i = 0; i < g_htmap_used; ++i)
      if (g_htmap_keys[i] == key) {
        *map = g_htmap_vals[i];
        return kStatusOk;
      }
  }
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return kStatusCuda;
  }
  cuuint64_t dims[5] = {static_cast<cuuint64_t>(cols), 16, static_cast<cuuint64_t>(slabs),
                        static_cast<cuuint64_t>(kv_heads), static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(st_row * 2), static_cast<cuuint64_t>(cols * 2),
                           static_cast<cuuint64_t>(st_head * 2), static_cast<cuuint64_t>(st_block * 2)};
  cuuint32_t box[5] = {static_cast<cuuint32_t>(cols), 16, static_cast<cuuint32_t>(slabs), 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapSwizzle sw = cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                           : (cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for the per-head cache", static_cast<int>(r));
    return kStatusCuda;
  }
  std::lock_guard<std::mutex> lock(g_tmap_mu);
  const int slot = g_htmap_used < 16 ? g_htmap_used++ : (g_htmap_next++ % 16);
  g_htmap_keys[slot] = key;
  g_htmap_vals[slot] = *map;
  return kStatusOk;
}

static int check_history_args(const HistoryArgs& a) {
  if (a.T < 0 || a.H < 1 || a.H > 16) {
    set_error("history attention needs 1..16 query heads per KV head (got H=%d, T=%d)", a.H, a.T);
    return kStatusInvalid;
  }
  if ((a.q_st % 2) || (a.q_sh % 2) || (reinterpret_cast<uintptr_t>(a.q) % 4)) {
    set_error("q_lat needs even token/head strides and a unit last-dim stride");
    return kStatusInvalid;
  }
  if (a.num_kv_splits < 1) {
    set_error("num_kv_splits must be >= 1");
    return kStatusInvalid;
  }
  if (a.page != 16 && a.page != 32) {
    set_error("page size %d unsupported (16 or 32)", a.page);
    return kStatusInvalid;
  }
  return kStatusOk;
}

static HistoryArgs make_history_args(const void* q, int64_t q_st, int64_t q_sh, const void* cache,
                                     int64_t num_blocks, int64_t st_block, int64_t st_row, const int32_t* bt,
                                     int64_t bt_st, int32_t max_blocks, const int32_t* ctx, int32_t T, int32_t H, int32_t W,
                                     int32_t page, float scale, int32_t splits, float* ws, int64_t ws_floats,
                                     int* err) {
  HistoryArgs a;
  a.q = q;
  a.q_st = q_st;
  a.q_sh = q_sh;
  a.cache = cache;
  a.num_blocks = num_blocks;
  a.cache_st_block = st_block;
  a.cache_st_row = st_row;
  a.block_table = bt;
  a.bt_st = bt_st;
  a.max_blocks = max_blocks;
  a.ctx = ctx;
  a.T = T;
  a.H = H;
  a.W = W;
  a.page = page;
  a.scale = scale;
  a.num_kv_splits = splits;
  a.ws = ws;
  a.ws_floats = ws_floats;
  a.waves = 1;
  a.err = err;
  return a;
}

}  // namespace hla

using namespace hla;

extern "C" {

int hla_s6_version(void) { return HLA_S6_ABI_VERSION; }

const char* hla_s6_last_error(void) { return g_error; }

uint64_t hla_s6_set_wait_limit_ns(uint64_t ns) {
  if (ns == 0) ns = 2000000000ull;
  return g_wait_ns.exchange(ns, std::memory_order_relaxed);
}

int hla_s6_history_attention(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                             int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row,
                             const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                             const int32_t* ctx, const uint8_t* empty, int32_t num_tokens, int32_t num_heads, int32_t width,
                             int32_t page, float scale, int32_t num_kv_splits, float* workspace,
                             int64_t workspace_floats, void* out, int64_t out_stride_t, int64_t out_stride_h,
                             float* lse, int* error_flag, void* stream) {
  HistoryArgs a = make_history_args(q_lat, q_stride_t, q_stride_h, cache, num_blocks, cache_stride_block,
                                    cache_stride_row, block_table, block_table_stride, max_blocks, ctx, num_tokens, num_heads,
                                    width, page, scale, num_kv_splits, workspace, workspace_floats, error_flag);
  int rc = check_history_args(a);
  if (rc) return rc;
  HistoryPlan plan;
  if ((rc = history_plan(a, &plan))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = history_split(a, plan, s))) return rc;
  return history_reduce(a, plan, empty, out, out_stride_t, out_stride_h, nullptr, lse, s);
}

int hla_s6_history_partials(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                            int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row,
                            const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                            const int32_t* ctx, int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page, float scale,
                            int32_t num_kv_splits, float* workspace, int64_t workspace_floats, int* error_flag,
                            int32_t flags, void* stream) {
  HistoryArgs a = make_history_args(q_lat, q_stride_t, q_stride_h, cache, num_blocks, cache_stride_block,
                                    cache_stride_row, block_table, block_table_stride, max_blocks, ctx, num_tokens, num_heads,
                                    width, page, scale, num_kv_splits, workspace, workspace_floats, error_flag);
  if (flags & ~HLA_S6_PARTIALS_AFTER_QUERY) {
    set_error("history partials: unknown flags 0x%x", flags);
    return kStatusInvalid;
  }
  a.pdl = (flags & HLA_S6_PARTIALS_AFTER_QUERY) != 0;
  int rc = check_history_args(a);
  if (rc) return rc;
  HistoryPlan plan;
  if ((rc = history_plan(a, &plan))) return rc;
  return history_split(a, plan, static_cast<cudaStream_t>(stream));
}

int hla_s6_history_reduce(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page,
                          int32_t num_kv_splits, float* workspace, int64_t workspace_floats, const uint8_t* empty,
                          void* out, int64_t out_stride_t, int64_t out_stride_h, float* out_f32, float* lse,
                          void* stream) {
  HistoryArgs a = make_history_args(nullptr, 0, 0, nullptr, 0, 0, 0, nullptr, 0, 0, nullptr, num_tokens, num_heads,
                                    width, page, 1.f, num_kv_splits, workspace, workspace_floats, nullptr);
  HistoryPlan plan;
  int rc = history_plan(a, &plan);
  if (rc) return rc;
  return history_reduce(a, plan, empty, out, out_stride_t, out_stride_h, out_f32, lse,
                        static_cast<cudaStream_t>(stream));
}

int hla_s6_history_attention_contig(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k,
                                    int64_t k_stride_b, int64_t k_stride_n, const void* v, int64_t v_stride_b,
                                    int64_t v_stride_n, const uint8_t* mask, int64_t mask_stride_b, int32_t batch,
                                    int32_t num_keys, int32_t num_heads, int32_t width, float scale,
                                    int32_t num_kv_splits, float* workspace, int64_t workspace_floats, void* z,
                                    int64_t z_stride_b, int64_t z_stride_h, float* z32, float* lse, int* error_flag,
                                    void* stream) {
  if (batch < 0 || num_heads < 1 || num_heads > 16 || num_keys < 1 || !mask || !lse) {
    set_error("contiguous history needs 1..16 heads, >= 1 key (a storage row), a mask and an lse output");
    return kStatusInvalid;
  }
  if ((q_stride_b % 2) || (q_stride_h % 2) || (reinterpret_cast<uintptr_t>(q) % 4) || (z_stride_b % 2) ||
      (z_stride_h % 2) || (reinterpret_cast<uintptr_t>(z) % 4) || (z32 && reinterpret_cast<uintptr_t>(z32) % 16)) {
    set_error("contiguous history: q / z need even strides and a unit last-dim stride, z32 16-byte alignment");
    return kStatusInvalid;
  }
  if (num_kv_splits < 1) {
    set_error("num_kv_splits must be >= 1");
    return kStatusInvalid;
  }
  ContigArgs c{};
  c.q = q;
  c.q_sb = q_stride_b;
  c.q_sh = q_stride_h;
  c.k = k;
  c.k_sb = k_stride_b;
  c.k_sn = k_stride_n;
  c.v = v;
  c.v_sb = v_stride_b;
  c.v_sn = v_stride_n;
  c.mask = mask;
  c.m_sb = mask_stride_b;
  c.B = batch;
  c.N = num_keys;
  c.H = num_heads;
  c.W = width;
  c.scale = scale;
  c.splits = num_kv_splits;
  c.ws = workspace;
  c.ws_floats = workspace_floats;
  c.z = z;
  c.z_sb = z_stride_b;
  c.z_sh = z_stride_h;
  c.z32 = z32;
  c.lse = lse;
  c.err = error_flag;
  return history_attention_contig(c, static_cast<cudaStream_t>(stream));
}

int hla_s6_history_reduce_exchange(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page,
                                   int32_t num_kv_splits, float* workspace, int64_t workspace_floats,
                                   const uint8_t* empty, uint64_t* const* parts, const int32_t* epoch,
                                   int32_t world, int32_t launch_flags, void* stream) {
  if (world < 1 || world > kMaxExchangeRanks || !parts || !epoch) {
    set_error("history reduce exchange needs 1..%d ranks, their part pointers and the slot's epoch counter",
              kMaxExchangeRanks);
    return kStatusInvalid;
  }
  ExchangeTargets x{};
  for (int d = 0; d < world; ++d) {
    if (!parts[d] || (reinterpret_cast<uintptr_t>(parts[d]) % 16)) {
      set_error("history reduce exchange: rank %d's part must be set and 16-byte aligned", d);
      return kStatusInvalid;
    }
    x.part[d] = parts[d];
  }
  x.epoch = epoch;
  x.world = world;
  HistoryArgs a = make_history_args(nullptr, 0, 0, nullptr, 0, 0, 0, nullptr, 0, 0, nullptr, num_tokens, num_heads,
                                    width, page, 1.f, num_kv_splits, workspace, workspace_floats, nullptr);
  HistoryPlan plan;
  int rc = history_plan(a, &plan);
  if (rc) return rc;
  return history_reduce_exchange(a, plan, empty, x, (launch_flags & HLA_S6_REDUCE_AFTER_PARTIALS) != 0,
                                 static_cast<cudaStream_t>(stream));
}

int hla_s6_history_plan(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t page, int32_t num_kv_splits,
                        int64_t workspace_floats, int32_t* stream_mode, int32_t* grid, int32_t* slots) {
  HistoryArgs a = make_history_args(nullptr, 0, 0, nullptr, 0, 0, 0, nullptr, 0, 0, nullptr, num_tokens, num_heads,
                                    width, page, 1.f, num_kv_splits, reinterpret_cast<float*>(0x100),
                                    workspace_floats, nullptr);
  HistoryPlan plan;
  int rc = history_plan(a, &plan);
  if (rc) return rc;
  if (stream_mode) *stream_mode = plan.stream_mode;
  if (grid) *grid = plan.grid;
  if (slots) *slots = plan.slots_cap;
  return kStatusOk;
}

}  // extern "C"
