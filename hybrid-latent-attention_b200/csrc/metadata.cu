// Integer step metadata of the S6 serving path, on the device: the per-token fields that
// s6_layer.StepContext derives once per step from vLLM's varlen metadata (s6_layer.py:52-70, with
// s6_ops.token_requests :61-68 and history_lengths :71-73), and the per-token gather of a
// per-request block table (StepContext.block_table, s6_layer.py:72-77).  The reference computes
// them with a chain of small torch ops (searchsorted, clamp, sub, where, index, comparisons); here
// one launch writes every field and one launch gathers a table.  All integer work, bit-exact.
#include "../../include/hla_s6.h"
#include "common.cuh"
#include "decode_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

constexpr int kMetaThreads = 256;

// Thread i < T handles token i; thread i < R also writes request i's history length.
__global__ void __launch_bounds__(kMetaThreads)
    step_metadata_kernel(const int32_t* __restrict__ qsl, int R, const int32_t* __restrict__ seq_lens, int T,
                         int window, int64_t* __restrict__ req_out, uint8_t* __restrict__ valid_out,
                         uint8_t* __restrict__ invalid_out, int32_t* __restrict__ hist_out,
                         int32_t* __restrict__ ctx_out, int32_t* __restrict__ ctx_lat_out,
                         uint8_t* __restrict__ empty_out, uint8_t* __restrict__ empty_lat_out) {
  const int i = blockIdx.x * kMetaThreads + threadIdx.x;
  if (i < R && hist_out) {
    const int h = seq_lens[i] - (qsl[i + 1] - qsl[i]);
    hist_out[i] = h > 0 ? h : 0;
  }
  if (i >= T) return;
  int r;
  const bool valid = token_request(qsl, R, i, r);
  if (req_out) req_out[i] = r;
  if (valid_out) valid_out[i] = valid;
  if (invalid_out) invalid_out[i] = !valid;
  if (!seq_lens) return;
  int c = 0;
  if (valid) {
    c = seq_lens[r] - (qsl[r + 1] - qsl[r]);
    c = c > 0 ? c : 0;
  }
  const int cl = window ? (c - window > 0 ? c - window : 0) : c;
  if (ctx_out) ctx_out[i] = c;
  if (ctx_lat_out) ctx_lat_out[i] = cl;
  if (empty_out) empty_out[i] = c == 0;
  if (empty_lat_out) empty_lat_out[i] = cl == 0;
}

// out[t, 0 .. cols) = table[req[t], 0 .. cols); a request index outside [0, R) gives a row of zeros.
// 16-byte copies when both rows are 16-byte aligned (VEC), else 4-byte copies.
template <bool VEC>
__global__ void __launch_bounds__(kMetaThreads)
    gather_rows_kernel(const int32_t* __restrict__ table, int64_t tab_st, int cols, int R,
                       const int64_t* __restrict__ req, int T, int32_t* __restrict__ out, int64_t out_st) {
  const int per_row = VEC ? cols / 4 : cols;
  const int64_t n = static_cast<int64_t>(T) * per_row;
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * kMetaThreads + threadIdx.x; k < n;
       k += static_cast<int64_t>(gridDim.x) * kMetaThreads) {
    const int t = static_cast<int>(k / per_row), j = static_cast<int>(k % per_row);
    const int64_t r = req[t];
    if constexpr (VEC) {
      int4 v = make_int4(0, 0, 0, 0);
      if (r >= 0 && r < R) v = reinterpret_cast<const int4*>(table + r * tab_st)[j];
      reinterpret_cast<int4*>(out + static_cast<int64_t>(t) * out_st)[j] = v;
    } else {
      out[static_cast<int64_t>(t) * out_st + j] = (r >= 0 && r < R) ? table[r * tab_st + j] : 0;
    }
  }
}

}  // namespace hla

using namespace hla;

extern "C" {

int hla_s6_step_metadata(const int32_t* query_start_loc, int32_t num_reqs, const int32_t* seq_lens,
                         int32_t num_tokens, int32_t window, int64_t* token_requests, uint8_t* valid,
                         uint8_t* invalid, int32_t* history, int32_t* ctx, int32_t* ctx_latent, uint8_t* empty,
                         uint8_t* empty_latent, void* stream) {
  if (num_reqs < 1 || num_tokens < 0 || window < 0 || !query_start_loc) {
    set_error("step metadata: needs query_start_loc with num_reqs >= 1 (got %d), num_tokens >= 0 (%d), window >= 0 "
              "(%d)", num_reqs, num_tokens, window);
    return kStatusInvalid;
  }
  if (!seq_lens && (history || ctx || ctx_latent || empty || empty_latent)) {
    set_error("step metadata: history lengths and ctx need seq_lens");
    return kStatusInvalid;
  }
  const int n = std::max(num_tokens, history ? num_reqs : 0);
  if (n == 0) return kStatusOk;
  step_metadata_kernel<<<(n + kMetaThreads - 1) / kMetaThreads, kMetaThreads, 0,
                         static_cast<cudaStream_t>(stream)>>>(query_start_loc, num_reqs, seq_lens, num_tokens, window,
                                                              token_requests, valid, invalid, history, ctx, ctx_latent,
                                                              empty, empty_latent);
  return cuda_status(cudaGetLastError(), "step_metadata_kernel launch");
}

int hla_s6_gather_block_table(const int32_t* table, int64_t table_stride, int32_t max_blocks, int32_t num_reqs,
                              const int64_t* token_requests, int32_t num_tokens, int32_t* out, int64_t out_stride,
                              void* stream) {
  // a row stride only matters between rows: a one-row table (or output) may carry any stride
  if (max_blocks < 0 || num_reqs < 0 || num_tokens < 0 || (num_reqs > 1 && table_stride < max_blocks) ||
      (num_tokens > 1 && out_stride < max_blocks)) {
    set_error("gather block table: bad sizes (max_blocks %d, num_reqs %d, num_tokens %d, strides %lld / %lld)",
              max_blocks, num_reqs, num_tokens, static_cast<long long>(table_stride),
              static_cast<long long>(out_stride));
    return kStatusInvalid;
  }
  if (num_tokens == 0 || max_blocks == 0) return kStatusOk;
  if (num_reqs <= 1) table_stride = max_blocks;
  if (num_tokens <= 1) out_stride = max_blocks;
  const bool vec = max_blocks % 4 == 0 && table_stride % 4 == 0 && out_stride % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(table) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const int64_t n = static_cast<int64_t>(num_tokens) * (vec ? max_blocks / 4 : max_blocks);
  const int grid = static_cast<int>(std::min<int64_t>((n + kMetaThreads - 1) / kMetaThreads, 1184));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec)
    gather_rows_kernel<true><<<grid, kMetaThreads, 0, s>>>(table, table_stride, max_blocks, num_reqs, token_requests,
                                                            num_tokens, out, out_stride);
  else
    gather_rows_kernel<false><<<grid, kMetaThreads, 0, s>>>(table, table_stride, max_blocks, num_reqs, token_requests,
                                                             num_tokens, out, out_stride);
  return cuda_status(cudaGetLastError(), "gather_rows_kernel launch");
}

}  // extern "C"
