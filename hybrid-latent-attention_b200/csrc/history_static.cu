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

// Device address of g_history_scratch in the current context.  In host code the symbol's name is a
// host-side stand-in, not a device address, so it is resolved with cudaGetSymbolAddress while that
// context is current, once per context, and kept.  The key is the CUDA context, not the device
// ordinal: after cudaDeviceReset, or with another context current on the same device, the array lives
// at another address and is looked up again.  The look-up may load this library's device code into
// the context, so the first call in each context must come before any stream capture.
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrent>(p);
  });
  return fn;
}

static int static_scratch(float** out) {
  constexpr int kSlots = 64;
  static std::mutex mu;
  static CUcontext ctxs[kSlots] = {nullptr};
  static float* addrs[kSlots] = {nullptr};
  static int used = 0, next = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "history_attention_static: cudaGetDevice");
  CtxGetCurrent get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get && get(&ctx) == CUDA_SUCCESS && !ctx) {
    // no context is current yet (the runtime makes the primary one current lazily): make it so now
    if ((e = cudaSetDevice(dev)) != cudaSuccess) return cuda_status(e, "history_attention_static: cudaSetDevice");
    get(&ctx);
  }
  if (!get || !ctx) {
    set_error("history_attention_static: no current CUDA context");
    return kStatusCuda;
  }
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (ctxs[i] == ctx) {
      *out = addrs[i];
      return kStatusOk;
    }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_history_scratch);
  if (e != cudaSuccess) return cuda_status(e, "history_attention_static: cudaGetSymbolAddress");
  const int slot = used < kSlots ? used++ : (next++ % kSlots);
  ctxs[slot] = ctx;
  addrs[slot] = static_cast<float*>(p);
  *out = addrs[slot];
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
