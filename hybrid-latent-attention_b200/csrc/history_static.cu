// History attention without a caller-provided workspace: hla_s6_history_attention_static.
//
// Who needs this: callers that cannot call cudaMalloc (or any allocating routine) when they run
// the op - for example a foreign-language host (a cgo / JNI / ctypes binding) that only receives
// device pointers for its inputs and outputs from the framework that owns GPU memory, or a
// serving process whose memory budget was reserved up front for KV caches, where an extra
// allocation in the middle of a request could fail.  They still pass inputs and outputs; the
// fp32 scratch the split kernel needs comes from the fixed array below instead.
//
// The array is a file-scope device variable of kStaticScratchFloats floats (8 MiB).  Every GPU
// that loads this library's code for it holds those 8 MiB until the process exits.  All calls
// share it: it keeps the previous call's contents, and two calls whose kernels overlap on the GPU
// (different streams, or different host threads, without ordering between them) race on it and
// corrupt each other's results.  Nothing in it needs to start at zero: each call writes every
// partial slot and slot map it later reads.
#include <mutex>

#include "../../include/hla_s6.h"
#include "hla_s6_internal.h"

namespace hla {

constexpr int64_t kStaticScratchFloats = int64_t(2) << 20;  // 2 Mi floats = 8 MiB

static __device__ __align__(256) float g_history_scratch[kStaticScratchFloats];

// Device address of g_history_scratch for the current device.  In host code the symbol's name is a
// host-side stand-in, not a device address, so it is resolved once per device with
// cudaGetSymbolAddress (with that device current) and cached.
static int static_scratch(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "history_attention_static: cudaGetDevice");
  if (dev < 0 || dev >= 64) {
    set_error("history_attention_static: device ordinal %d out of range", dev);
    return kStatusInvalid;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_history_scratch);
    if (e != cudaSuccess) return cuda_status(e, "history_attention_static: cudaGetSymbolAddress");
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return kStatusOk;
}

}  // namespace hla

using namespace hla;

extern "C" int hla_s6_history_attention_static(const void* q_lat, int64_t q_stride_t, int64_t q_stride_h,
                                               const void* cache, int64_t num_blocks, int64_t cache_stride_block,
                                               int64_t cache_stride_row, const int32_t* block_table,
                                               int64_t block_table_stride, int32_t max_blocks, const int32_t* ctx,
                                               const uint8_t* empty, int32_t num_tokens, int32_t num_heads,
                                               int32_t width, int32_t page, float scale, int32_t num_kv_splits,
                                               void* out, int64_t out_stride_t, int64_t out_stride_h, float* lse,
                                               int* error_flag, void* stream) {
  const int64_t need = static_cast<int64_t>(num_tokens) * num_kv_splits * num_heads * (width + 1);
  if (num_tokens < 0 || num_kv_splits < 1 || num_heads < 1 || width < 1) {
    set_error("history_attention_static: bad sizes (T=%d, splits=%d, H=%d, W=%d)", num_tokens, num_kv_splits,
              num_heads, width);
    return kStatusInvalid;
  }
  if (need > kStaticScratchFloats) {
    set_error("history_attention_static: T * num_kv_splits * H * (W + 1) = %lld floats exceeds the %lld-float "
              "static scratch; use fewer splits or hla_s6_history_attention with a caller workspace",
              static_cast<long long>(need), static_cast<long long>(kStaticScratchFloats));
    return kStatusOverflow;
  }
  float* scratch = nullptr;
  int rc = static_scratch(&scratch);
  if (rc) return rc;
  return hla_s6_history_attention(q_lat, q_stride_t, q_stride_h, cache, num_blocks, cache_stride_block,
                                  cache_stride_row, block_table, block_table_stride, max_blocks, ctx, empty,
                                  num_tokens, num_heads, width, page, scale, num_kv_splits, scratch, need, out,
                                  out_stride_t, out_stride_h, lse, error_flag, stream);
}
