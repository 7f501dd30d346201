// Fused decode combine for one (layer, loop) of the S6 decode step: the tail of
// s6_layer.attend's decode branch (s6_layer.py:97-115) in one launch:
//   1. reduce the history kernel's split partials -> z[t, h, :] (bf16 values, as the
//      reference's history output o_hist is bf16) and lse_hist      (vLLM stage 2, s6_ops.py:158)
//   2. exact window over keys [pos - W, pos] of this loop's exact cache  (window_attention_fa, :317)
//   3. up-projection o_hist = z . B[h]  (bf16 result)                     (einsum, s6_layer.py:114)
//   4. LSE merge, invalid (padding) tokens zeroed                        (merge_states, s6_ops.py:262)
// CTA = (4 tokens, 1 head), 4 warps: warp w owns token t0 + w in steps 1-2; thread d owns output
// column d in steps 3-4.  Instead of split partials the kernel can take an already reduced
// (z fp32 [T,H,W], lse [H,T]) pair, which is how a sequence-split history arrives after its
// cross-GPU exchange.
#include "combine.cuh"
#include "common.cuh"
#include "decode_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

template <int W>
__global__ void __launch_bounds__(128) decode_combine_kernel(const CombineParams p) {
  constexpr int TT = 4, D = 128;
  __shared__ float z_s[TT][W];
  __shared__ float q_s[TT][D];
  __shared__ float ow_s[TT][D];
  __shared__ float lh_s[TT], lw_s[TT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * TT, h = blockIdx.y, T = p.T, H = p.H;

  // ---- 1. history: reduce partials (or take the pre-reduced pair)
  {
    const int t = t0 + warp;
    float lse_h = -INFINITY;
    constexpr int NV = W / 128;  // float4 per lane
    float4 acc[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < T && !(p.empty && p.empty[t])) {
      if (p.z_in) {
        lse_h = p.lse_in[static_cast<int64_t>(h) * T + t];
        if (lse_h != -INFINITY) {
          const float4* src = reinterpret_cast<const float4*>(p.z_in + (static_cast<int64_t>(t) * H + h) * W);
#pragma unroll
          for (int i = 0; i < NV; ++i) acc[i] = src[i * 32 + lane];
        }
      } else {
        int lo = t, hi = t + 1;
        if (p.stream_mode) {
          const int2 m = p.meta[t];
          lo = m.x;
          hi = m.y;
        }
        float mx = -INFINITY;
        for (int s = lo; s < hi; ++s) mx = fmaxf(mx, p.ws_lse[static_cast<int64_t>(s) * H + h]);
        if (mx != -INFINITY) {
          float wsum = 0.f;
          for (int s = lo; s < hi; ++s) {
            const float wgt = expf(p.ws_lse[static_cast<int64_t>(s) * H + h] - mx);
            wsum += wgt;
            const float4* src = reinterpret_cast<const float4*>(p.ws_o + (static_cast<int64_t>(s) * H + h) * W);
#pragma unroll
            for (int i = 0; i < NV; ++i) {
              const float4 v = src[i * 32 + lane];
              acc[i].x += wgt * v.x; acc[i].y += wgt * v.y; acc[i].z += wgt * v.z; acc[i].w += wgt * v.w;
            }
          }
          const float inv = 1.f / wsum;
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            acc[i].x *= inv; acc[i].y *= inv; acc[i].z *= inv; acc[i].w *= inv;
          }
          lse_h = mx + logf(wsum);
        }
      }
    }
    if (lse_h == -INFINITY) {
#pragma unroll
      for (int i = 0; i < NV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int d = (i * 32 + lane) * 4;
      z_s[warp][d + 0] = bf16_round(acc[i].x);
      z_s[warp][d + 1] = bf16_round(acc[i].y);
      z_s[warp][d + 2] = bf16_round(acc[i].z);
      z_s[warp][d + 3] = bf16_round(acc[i].w);
    }
    if (lane == 0) lh_s[warp] = lse_h;

    // ---- 2. exact window of this token (o rounded to bf16 as the FA output is)
    float o[4], lse_w;
    if (t < T) {
      window_warp(p.win, t, h, q_s[warp], o, lse_w);
    } else {
      o[0] = o[1] = o[2] = o[3] = 0.f;
      lse_w = -INFINITY;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) ow_s[warp][lane * 4 + e] = bf16_round(o[e]);
    if (lane == 0) lw_s[warp] = lse_w;
  }
  __syncthreads();

  // ---- 3. up-projection: thread d, four tokens
  const int d = threadIdx.x;
  float acc[TT] = {0.f, 0.f, 0.f, 0.f};
  const __nv_bfloat16* Bh = p.B + static_cast<int64_t>(h) * p.b_sh + d;
#pragma unroll 8
  for (int k = 0; k < W; ++k) {
    const float b = __bfloat162float(Bh[static_cast<int64_t>(k) * p.b_sk]);
#pragma unroll
    for (int tt = 0; tt < TT; ++tt) acc[tt] = fmaf(z_s[tt][k], b, acc[tt]);
  }

  // ---- 4. merge
#pragma unroll
  for (int tt = 0; tt < TT; ++tt) {
    const int t = t0 + tt;
    if (t >= T) break;
    const bool invalid = t >= p.win.qsl[p.win.R];
    float w1, w2;
    merge_weights_states(lh_s[tt], lw_s[tt], w1, w2);
    const float r = invalid ? 0.f : bf16_round(acc[tt]) * w1 + ow_s[tt][d] * w2;
    p.out[static_cast<int64_t>(t) * p.o_st + static_cast<int64_t>(h) * p.o_sh + d] = __float2bfloat16_rn(r);
    if (d == 0 && p.lse_out) {
      float l1 = lh_s[tt], l2 = lw_s[tt];
      p.lse_out[static_cast<int64_t>(h) * T + t] = invalid ? -INFINITY : merged_lse(l1, l2);
    }
  }
}

int decode_combine(const CombineParams& p, int W, cudaStream_t s) {
  if (p.T == 0) return kStatusOk;
  dim3 grid((p.T + 3) / 4, p.H);
  switch (W) {
    case 256: decode_combine_kernel<256><<<grid, 128, 0, s>>>(p); break;
    case 512: decode_combine_kernel<512><<<grid, 128, 0, s>>>(p); break;
    default: set_error("decode combine width %d unsupported (256 or 512)", W); return kStatusInvalid;
  }
  return cuda_status(cudaGetLastError(), "decode_combine_kernel launch");
}

}  // namespace hla
