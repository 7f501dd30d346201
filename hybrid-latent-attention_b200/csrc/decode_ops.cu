// The per-(layer, loop) S6 decode ops around the history reader:
//   A5  exact window (window_attention_fa)          s6_ops.py:317-331
//   A7  LSE merges (merge_states / merge_lse)       s6_ops.py:262-284, 353-361
//   A4  latent RoPE (in place)                      s6_ops.py:23-41
//   A10 exact-cache append with exact RoPE          ouro_latent.py:113-123
//   A9+A10 committed row: latent RoPE + paged scatter  s6_layer.py:135-147, ouro_latent.py:127-129
// (the writer projection and the latent query GEMMs live in gemm_ops.cu)
//
// Latent RoPE everywhere follows the torch bf16 operation order of LatentLayer.pack
// (register.py:73-79): bf16(x*c), bf16(rotate_half(x)*s), bf16(sum), so committed cache rows
// are bit-identical to the reference's packed rows given the same register values.
#include "common.cuh"
#include "decode_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

// -------------------------------------------------------------------- A5 exact window
__global__ void __launch_bounds__(128) window_kernel(const WindowArgs a, __nv_bfloat16* __restrict__ out,
                                                     int64_t o_st, int64_t o_sh, float* __restrict__ lse_out, int T,
                                                     int H) {
  __shared__ float q_s[4][128];
  __shared__ int32_t qsl_s[kQslCap];
  __shared__ __align__(16) uint8_t v_s[4][kWindowVBytes];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x, h = blockIdx.y * 4 + warp;
  WindowArgs w = a;
  if (!a.ctx_tok) w.qsl = stage_qsl(a.qsl, a.R, qsl_s);
  if (h >= H) return;
  float o[4], lse;
  if (!w.ctx_tok && w.window <= 32) window_warp_short(w, t, h, q_s[warp], v_s[warp], o, lse);
  else window_warp(w, t, h, q_s[warp], o, lse);
  __nv_bfloat16* dst = out + static_cast<int64_t>(t) * o_st + static_cast<int64_t>(h) * o_sh + lane * 4;
  reinterpret_cast<__nv_bfloat162*>(dst)[0] = __floats2bfloat162_rn(o[0], o[1]);
  reinterpret_cast<__nv_bfloat162*>(dst)[1] = __floats2bfloat162_rn(o[2], o[3]);
  if (lane == 0) lse_out[static_cast<int64_t>(h) * T + t] = lse;
}

int window_attention(const WindowArgs& a, int T, int H, void* out, int64_t o_st, int64_t o_sh, float* lse,
                     cudaStream_t s) {
  if (T == 0) return kStatusOk;
  dim3 grid(T, (H + 3) / 4);
  window_kernel<<<grid, 128, 0, s>>>(a, static_cast<__nv_bfloat16*>(out), o_st, o_sh, lse, T, H);
  return cuda_status(cudaGetLastError(), "window_kernel launch");
}

// -------------------------------------------------------------------- A7 merges
// mode 0: merge_states (+inf counts as empty, invalid rows zeroed);  mode 1: merge_lse.
__global__ void merge_kernel(const __nv_bfloat16* __restrict__ o1, int64_t s1t, int64_t s1h,
                             const float* __restrict__ lse1, const __nv_bfloat16* __restrict__ o2, int64_t s2t,
                             int64_t s2h, const float* __restrict__ lse2, const uint8_t* __restrict__ invalid,
                             __nv_bfloat16* __restrict__ out, int64_t sot, int64_t soh, float* __restrict__ lse_out,
                             int T, int H, int D, int mode) {
  const int t = blockIdx.x, h = blockIdx.y;
  float l1 = lse1[static_cast<int64_t>(h) * T + t], l2 = lse2[static_cast<int64_t>(h) * T + t];
  float w1, w2;
  if (mode == 0) merge_weights_states(l1, l2, w1, w2);
  else merge_weights_lse(l1, l2, w1, w2);
  const bool zero = mode == 0 && invalid && invalid[t];
  const __nv_bfloat16* a = o1 + static_cast<int64_t>(t) * s1t + static_cast<int64_t>(h) * s1h;
  const __nv_bfloat16* b = o2 + static_cast<int64_t>(t) * s2t + static_cast<int64_t>(h) * s2h;
  __nv_bfloat16* c = out + static_cast<int64_t>(t) * sot + static_cast<int64_t>(h) * soh;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float x = __bfloat162float(a[d]), y = __bfloat162float(b[d]);
    if (mode == 1) {  // merge_lse: nan_to_num on both inputs (FA scratch rows)
      x = isnan(x) ? 0.f : (isinf(x) ? copysignf(3.4028234663852886e38f, x) : x);
      y = isnan(y) ? 0.f : (isinf(y) ? copysignf(3.4028234663852886e38f, y) : y);
    }
    const float r = zero ? 0.f : x * w1 + y * w2;
    c[d] = __float2bfloat16_rn(r);
  }
  if (threadIdx.x == 0 && lse_out) lse_out[static_cast<int64_t>(h) * T + t] = merged_lse(l1, l2);
}

int merge(const void* o1, int64_t s1t, int64_t s1h, const float* lse1, const void* o2, int64_t s2t, int64_t s2h,
          const float* lse2, const uint8_t* invalid, void* out, int64_t sot, int64_t soh, float* lse_out, int T, int H,
          int D, int mode, cudaStream_t s) {
  if (T == 0) return kStatusOk;
  dim3 grid(T, H);
  merge_kernel<<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(o1), s1t, s1h, lse1,
                                    static_cast<const __nv_bfloat16*>(o2), s2t, s2h, lse2, invalid,
                                    static_cast<__nv_bfloat16*>(out), sot, soh, lse_out, T, H, D, mode);
  return cuda_status(cudaGetLastError(), "merge_kernel launch");
}

// -------------------------------------------------------------------- A4 latent RoPE (in place)
__global__ void latent_rope_kernel(__nv_bfloat16* __restrict__ x, int64_t st, int64_t sh, int H, int w,
                                   const int64_t* __restrict__ positions, const __nv_bfloat16* __restrict__ table,
                                   int64_t tab_st, int64_t max_pos) {
  const int t = blockIdx.x;
  const int64_t pos = clamp_pos(positions[t], max_pos);
  const __nv_bfloat16* row = table + pos * tab_st;
  const int half = w >> 1;
  for (int idx = threadIdx.x; idx < H * half; idx += blockDim.x) {
    const int h = idx / half, i = idx - h * half;
    __nv_bfloat16* p = x + static_cast<int64_t>(t) * st + static_cast<int64_t>(h) * sh;
    float a, b;
    rope_pair_torch(__bfloat162float(p[i]), __bfloat162float(p[i + half]), __bfloat162float(row[i]),
                    __bfloat162float(row[half + i]), a, b);
    p[i] = __float2bfloat16_rn(a);
    p[i + half] = __float2bfloat16_rn(b);
  }
}

int latent_rope(void* x, int64_t st, int64_t sh, int T, int H, int w, const int64_t* positions, const void* table,
                int64_t tab_st, int64_t max_pos, cudaStream_t s) {
  if (T == 0) return kStatusOk;
  latent_rope_kernel<<<T, 256, 0, s>>>(static_cast<__nv_bfloat16*>(x), st, sh, H, w, positions,
                                       static_cast<const __nv_bfloat16*>(table), tab_st, max_pos);
  return cuda_status(cudaGetLastError(), "latent_rope_kernel launch");
}

// -------------------------------------------------------------------- A10 exact append
// Exact neox RoPE (fp32 math, one rounding, as vLLM's rotary_embedding) of q (in place) and k,
// then k_rope | v into the exact cache at slot = block_table[req, pos // page] * page + pos % page.
__global__ void __launch_bounds__(256) exact_append_kernel(const ExactArgs a) {
  const int t = blockIdx.x;
  int r;
  const bool valid = token_request(a.qsl, a.R, t, r);
  const int64_t pos = a.positions[t];
  const int64_t pc = clamp_pos(pos, a.max_pos);
  const float* cs = a.cos_sin + pc * a.cs_st;  // [cos 64 | sin 64]
  int64_t slot = -1;
  if (valid && pos >= 0) {
    const int64_t col = pos / a.page;
    if (col < a.max_blocks) {
      const int blk = a.bt[static_cast<int64_t>(r) * a.bt_st + col];
      slot = static_cast<int64_t>(blk) * a.page + pos % a.page;
    }
  }
  if (a.slot_out && threadIdx.x == 0) a.slot_out[t] = slot;
  const int H = a.H;
  for (int idx = threadIdx.x; idx < H * 64; idx += blockDim.x) {
    const int h = idx >> 6, i = idx & 63;
    const float c = cs[i], s = cs[64 + i];
    if (a.q) {
      __nv_bfloat16* qp = a.q + static_cast<int64_t>(t) * a.q_st + static_cast<int64_t>(h) * a.q_sh;
      const float x1 = __bfloat162float(qp[i]), x2 = __bfloat162float(qp[i + 64]);
      qp[i] = __float2bfloat16_rn(x1 * c - x2 * s);
      qp[i + 64] = __float2bfloat16_rn(x2 * c + x1 * s);
    }
    const __nv_bfloat16* kp = a.k + static_cast<int64_t>(t) * a.k_st + static_cast<int64_t>(h) * a.k_sh;
    const float k1 = __bfloat162float(kp[i]), k2 = __bfloat162float(kp[i + 64]);
    const __nv_bfloat16 kr1 = __float2bfloat16_rn(k1 * c - k2 * s), kr2 = __float2bfloat16_rn(k2 * c + k1 * s);
    if (a.k_out) {
      __nv_bfloat16* ko = a.k_out + static_cast<int64_t>(t) * a.ko_st + static_cast<int64_t>(h) * a.ko_sh;
      ko[i] = kr1;
      ko[i + 64] = kr2;
    }
    if (slot >= 0 && slot / a.page < a.num_blocks) {
      const __nv_bfloat16* vp = a.v + static_cast<int64_t>(t) * a.v_st + static_cast<int64_t>(h) * a.v_sh;
      __nv_bfloat16* row = a.cache + (slot / a.page) * a.c_sb + static_cast<int64_t>(h) * a.c_sh +
                           (slot % a.page) * a.c_sr;
      row[i] = kr1;
      row[i + 64] = kr2;
      row[128 + i] = vp[i];
      row[128 + i + 64] = vp[i + 64];
    }
  }
}

int exact_append(const ExactArgs& a, int T, cudaStream_t s) {
  if (T == 0) return kStatusOk;
  exact_append_kernel<<<T, 256, 0, s>>>(a);
  return cuda_status(cudaGetLastError(), "exact_append_kernel launch");
}

// -------------------------------------------------------------------- A9 + A10 committed row
// row [T, 2w] (K | V) -> cache slot: K half latent-RoPE'd (torch bf16 order), V half copied.
__global__ void commit_kernel(const CommitArgs a) {
  const int t = blockIdx.x;
  int r;
  const bool valid = token_request(a.qsl, a.R, t, r);
  const int64_t pos = a.positions[t];
  int64_t slot = -1;
  if (valid && pos >= 0) {
    const int64_t col = pos / a.page;
    if (col < a.max_blocks) slot = static_cast<int64_t>(a.bt[static_cast<int64_t>(r) * a.bt_st + col]) * a.page + pos % a.page;
  }
  if (a.slot_out && threadIdx.x == 0) a.slot_out[t] = slot;
  if (slot < 0 || slot / a.page >= a.num_blocks) return;
  const int w = a.w, half = w >> 1;
  const __nv_bfloat16* src = a.row + static_cast<int64_t>(t) * a.row_st;
  __nv_bfloat16* dst = a.cache + (slot / a.page) * a.c_sb + (slot % a.page) * a.c_sr;
  const __nv_bfloat16* tab = a.table + clamp_pos(pos, a.max_pos) * a.tab_st;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float x, y;
    rope_pair_torch(__bfloat162float(src[i]), __bfloat162float(src[i + half]), __bfloat162float(tab[i]),
                    __bfloat162float(tab[half + i]), x, y);
    dst[i] = __float2bfloat16_rn(x);
    dst[i + half] = __float2bfloat16_rn(y);
  }
  for (int i = threadIdx.x; i < w; i += blockDim.x) dst[w + i] = src[w + i];
}

int commit_rows(const CommitArgs& a, int T, cudaStream_t s) {
  if (T == 0) return kStatusOk;
  commit_kernel<<<T, 256, 0, s>>>(a);
  return cuda_status(cudaGetLastError(), "commit_kernel launch");
}

}  // namespace hla
