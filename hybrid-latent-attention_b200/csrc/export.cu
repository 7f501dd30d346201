// Rollout cache export gather (hla/vllm_latent/cache_export.py:160-174): the latent rows of one
// finished request, positions 0 .. length-1 of every layer's main and loop-1 paged caches, into one
// contiguous [layers, length, main_w + l1_w] buffer (main | l1 per row), ready for a single
// device-to-host copy.  Physical rows come from each kv group's block list exactly as the exporter
// indexes them: block = blocks[pos / block_size], row = pos % block_size.
//
// HBM-bound byte copy: one warp per (layer, position) row, 16-byte loads and stores, grid
// (row chunks, layers).  A block id outside the cache records an error code in the device error
// word and leaves that row zeroed (the reference's indexing would raise).
#include "../../include/hla_s6.h"
#include "common.cuh"
#include "hla_s6_internal.h"

namespace hla {

constexpr int kExportMaxLayers = 64;
constexpr int kExportWarps = 8;

struct ExportArgs {
  const __nv_bfloat16* main[kExportMaxLayers];
  const __nv_bfloat16* l1[kExportMaxLayers];
  int layers;
  int64_t main_sb, main_sr, l1_sb, l1_sr;  // element strides per block / row (same for every layer)
  int main_w, l1_w;                        // elements per row (multiples of 8)
  int main_bs, l1_bs;                      // block sizes of the two kv groups
  const int32_t* main_blocks;              // physical block lists of the request
  const int32_t* l1_blocks;
  int64_t main_nb, l1_nb;                  // blocks in each cache (bounds)
  int64_t length;
  __nv_bfloat16* out;                      // [layers, length, main_w + l1_w]
  int* err;
};

__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int n16, int lane) {
  for (int i = lane; i < n16; i += 32) dst[i] = __ldg(src + i);
}
__device__ __forceinline__ void zero_row(uint4* __restrict__ dst, int n16, int lane) {
  for (int i = lane; i < n16; i += 32) dst[i] = make_uint4(0u, 0u, 0u, 0u);
}

__global__ void __launch_bounds__(kExportWarps * 32) export_rows_kernel(const ExportArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int layer = blockIdx.y;
  const int64_t pos = static_cast<int64_t>(blockIdx.x) * kExportWarps + warp;
  if (pos >= a.length || layer >= a.layers) return;
  const int row_w = a.main_w + a.l1_w;
  uint4* dst = reinterpret_cast<uint4*>(a.out + (static_cast<int64_t>(layer) * a.length + pos) * row_w);
  {
    const int64_t blk = a.main_blocks[pos / a.main_bs];
    if (blk < 0 || blk >= a.main_nb) {
      if (lane == 0) record_error(a.err, kErrSlots);
      zero_row(dst, a.main_w / 8, lane);
    } else {
      const __nv_bfloat16* src = a.main[layer] + blk * a.main_sb + (pos % a.main_bs) * a.main_sr;
      copy_row(dst, reinterpret_cast<const uint4*>(src), a.main_w / 8, lane);
    }
  }
  {
    uint4* d = dst + a.main_w / 8;
    const int64_t blk = a.l1_blocks[pos / a.l1_bs];
    if (blk < 0 || blk >= a.l1_nb) {
      if (lane == 0) record_error(a.err, kErrSlots);
      zero_row(d, a.l1_w / 8, lane);
    } else {
      const __nv_bfloat16* src = a.l1[layer] + blk * a.l1_sb + (pos % a.l1_bs) * a.l1_sr;
      copy_row(d, reinterpret_cast<const uint4*>(src), a.l1_w / 8, lane);
    }
  }
}

}  // namespace hla

using namespace hla;

extern "C" int hla_s6_export_rows(const void* const* main_caches, const void* const* l1_caches, int32_t num_layers,
                                  int64_t main_num_blocks, int64_t main_stride_block, int64_t main_stride_row,
                                  int32_t main_width, int32_t main_block_size, const int32_t* main_blocks, int64_t main_blocks_len,
                                  int64_t l1_num_blocks, int64_t l1_stride_block, int64_t l1_stride_row,
                                  int32_t l1_width, int32_t l1_block_size, const int32_t* l1_blocks, int64_t l1_blocks_len, int64_t length,
                                  void* out, int* error_flag, void* stream) {
  if (num_layers < 1 || num_layers > kExportMaxLayers || !main_caches || !l1_caches || !out || !main_blocks ||
      !l1_blocks || length < 0) {
    set_error("export: 1..%d layers, their caches, both block lists and an output are required", kExportMaxLayers);
    return kStatusInvalid;
  }
  if ((main_width % 8) || (l1_width % 8) || (main_stride_block % 8) || (main_stride_row % 8) ||
      (l1_stride_block % 8) || (l1_stride_row % 8) || main_block_size < 1 || l1_block_size < 1 ||
      (reinterpret_cast<uintptr_t>(out) % 16)) {
    set_error("export: widths and strides must be multiples of 8 elements, block sizes >= 1, out 16-byte aligned");
    return kStatusInvalid;
  }
  if ((length + main_block_size - 1) / main_block_size > main_blocks_len ||
      (length + l1_block_size - 1) / l1_block_size > l1_blocks_len) {
    set_error("export: the block lists (%lld main, %lld loop-1) do not cover %lld positions",
              static_cast<long long>(main_blocks_len), static_cast<long long>(l1_blocks_len),
              static_cast<long long>(length));
    return kStatusInvalid;
  }
  ExportArgs a{};
  for (int l = 0; l < num_layers; ++l) {
    if (!main_caches[l] || !l1_caches[l] || (reinterpret_cast<uintptr_t>(main_caches[l]) % 16) ||
        (reinterpret_cast<uintptr_t>(l1_caches[l]) % 16)) {
      set_error("export: layer %d's caches must be set and 16-byte aligned", l);
      return kStatusInvalid;
    }
    a.main[l] = static_cast<const __nv_bfloat16*>(main_caches[l]);
    a.l1[l] = static_cast<const __nv_bfloat16*>(l1_caches[l]);
  }
  a.layers = num_layers;
  a.main_sb = main_stride_block;
  a.main_sr = main_stride_row;
  a.l1_sb = l1_stride_block;
  a.l1_sr = l1_stride_row;
  a.main_w = main_width;
  a.l1_w = l1_width;
  a.main_bs = main_block_size;
  a.l1_bs = l1_block_size;
  a.main_blocks = main_blocks;
  a.l1_blocks = l1_blocks;
  a.main_nb = main_num_blocks;
  a.l1_nb = l1_num_blocks;
  a.length = length;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.err = error_flag;
  if (length == 0) return kStatusOk;
  dim3 grid(static_cast<unsigned>((length + kExportWarps - 1) / kExportWarps), num_layers);
  export_rows_kernel<<<grid, kExportWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cuda_status(cudaGetLastError(), "export_rows_kernel launch");
}
