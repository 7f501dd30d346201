// Internal host-side interfaces shared by the S6 kernel translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace hla {

enum Status : int {
  kStatusOk = 0,
  kStatusInvalid = 1,   // bad shape / stride / dtype: ValueError on the Python side
  kStatusOverflow = 2,  // workspace too small: RuntimeError
  kStatusCuda = 3,      // CUDA runtime / driver failure: RuntimeError
};

// Rows above this count use one CTA per row instead of the stream-K page split.
constexpr int kHistoryMaxStreamRows = 1024;

void set_error(const char* fmt, ...);
// Bound (device ns) that launches give their kernels' mbarrier and peer-flag waits
// (hla_s6_set_wait_limit_ns; kDefaultWaitNs until set).
uint64_t wait_limit_ns();

// Raise `func`'s dynamic shared-memory limit to `bytes`, once per device (bit `dev` of `mask`).
template <typename F>
inline void ensure_smem_limit(F func, int bytes, unsigned& mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(mask & (1u << dev))) {
    cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    mask |= 1u << dev;
  }
}
int cuda_status(cudaError_t e, const char* what);

// 4-D TMA descriptor over a paged latent cache [num_blocks, 1, page, 2W] (unit last stride):
// dims (64 columns, page rows, 2W/64 slabs, blocks) with SWIZZLE_128B, so a box of
// (64, page, 2W/64, 1) is one whole page laid out [slab][row][64] in shared memory.
int latent_cache_tmap(CUtensorMap* map, const void* cache, int64_t num_blocks, int64_t st_block, int64_t st_row,
                      int W, int page);

// cuCtxGetCurrent through the runtime's driver entry point (null when unavailable): the CUDA context
// that device-symbol addresses belong to (history_static.cu).
using CtxGetCurrent = CUresult (*)(CUcontext*);
CtxGetCurrent ctx_get_current();

struct HistoryArgs {
  const void* q;            // bf16 [T, H, W], unit last stride
  int64_t q_st, q_sh;
  const void* cache;        // bf16 [num_blocks, 1, page, 2W]
  int64_t num_blocks, cache_st_block, cache_st_row;
  const int32_t* block_table;
  int64_t bt_st;
  int32_t max_blocks;
  const int32_t* ctx;
  int32_t T, H, W, page;
  float scale;
  int32_t num_kv_splits;
  float* ws;
  int64_t ws_floats;
  int32_t waves;            // CTAs per SM slot multiplier for the stream-K grid (>= 1)
  int* err;
  int32_t pdl = 0;          // launch the split as a programmatic dependent of the preceding launch
};

struct HistoryPlan {
  int stream_mode;
  int grid;
  int slots_cap;
  float* ws_o;
  float* ws_lse;
  int2* meta;
};

int history_plan(const HistoryArgs& a, HistoryPlan* plan);
int history_split(const HistoryArgs& a, const HistoryPlan& plan, cudaStream_t stream);
int history_reduce_strided(const HistoryArgs& a, const HistoryPlan& plan, const uint8_t* empty, void* out,
                           int64_t o_st, int64_t o_sh, float* out_f32, float* lse, int64_t lse_st, int64_t lse_sh,
                           cudaStream_t stream);

// Contiguous-layout reader (fused_history.history_attention): q [B, H, W], K / V [B, N, W] (row
// strides k_sb / k_sn ...), mask [B, N] (uint8), outputs z bf16 [B, H, W] (strided), z32 fp32
// [B, H, W] contiguous (optional), lse fp32 [B, H].
struct ContigArgs {
  const void* q;
  int64_t q_sb, q_sh;
  const void* k;
  int64_t k_sb, k_sn;
  const void* v;
  int64_t v_sb, v_sn;
  const uint8_t* mask;
  int64_t m_sb;
  int B, N, H, W;
  float scale;
  int splits;
  float* ws;
  int64_t ws_floats;
  void* z;
  int64_t z_sb, z_sh;
  float* z32;
  float* lse;
  int* err;
};
int history_attention_contig(const ContigArgs& c, cudaStream_t stream);
// 4-D TMA map over the combine's up-projection B [H, W, 128] bf16 (capi.cu).
int combine_b_tmap(CUtensorMap* map, const void* B, int H, int W, int64_t b_sh, int64_t b_sk);
// 5-D TMA map over a per-head cache [num_blocks, kv_heads, 16, >= Lk] from column 0 of `base` (capi.cu):
// a box is `slabs` slabs of `cols` columns (64, 32 or 16) of one page of one KV head, laid out
// [slab][row][2 * cols bytes] with the (2 * cols)-byte swizzle.
int heads_cache_tmap(CUtensorMap* map, const void* base, int64_t num_blocks, int64_t kv_heads, int64_t st_block,
                     int64_t st_head, int64_t st_row, int cols, int slabs);
// 4-D TMA map over a [B, N, W] bf16 tensor: (64, N, W/64, B) with boxes of `tile` rows (capi.cu).
int contig_rows_tmap(CUtensorMap* map, const void* base, int64_t B, int64_t N, int W, int64_t st_b, int64_t st_n,
                     int tile);

// Targets of the fused sequence-split exchange (history_reduce_exchange): this rank's part - exchange
// words z [T, H, W] then lse [H, T] - in every rank's receive slot, and the slot's local use counter
// (the words carry the tag epoch + 1).
constexpr int kMaxExchangeRanks = 8;
struct ExchangeTargets {
  uint64_t* part[kMaxExchangeRanks];
  const int* epoch;
  int world;
};
// pdl: launch as a programmatic dependent of the immediately preceding launch (the history split).
int history_reduce_exchange(const HistoryArgs& a, const HistoryPlan& plan, const uint8_t* empty,
                            const ExchangeTargets& x, bool pdl, cudaStream_t stream);
int history_reduce(const HistoryArgs& a, const HistoryPlan& plan, const uint8_t* empty, void* out, int64_t o_st,
                   int64_t o_sh, float* out_f32, float* lse, cudaStream_t stream);

}  // namespace hla
