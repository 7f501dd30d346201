// Fused decode combine for one (layer, loop) of the S6 decode step: the tail of
// s6_layer.attend's decode branch (s6_layer.py:97-115) in one launch:
//   1. reduce the history kernel's split partials -> z[t, h, :] (rounded to bf16, as the
//      reference's history output o_hist is bf16) and lse_hist      (vLLM stage 2, s6_ops.py:158)
//   2. exact window over keys [pos - W, pos] of this loop's exact cache  (window_attention_fa, :317)
//   3. up-projection o_hist = z . B[h] (bf16 result)                      (einsum, s6_layer.py:114)
//   4. LSE merge, invalid (padding) tokens zeroed                        (merge_states, s6_ops.py:262)
// CTA = (8 tokens, head h), 8 warps, one token per warp.  All of B[h] ([W, 128] bf16) is put in
// flight with cp.async before steps 1-2, so its latency hides behind them; step 3 is mma.m16n8k16 with the 8
// tokens as M (rows 8-15 zero; z from shared memory, B via ldmatrix.trans).
// With an external exact part (chunk_o) and more CTAs than one wave fills, a CTA takes 16 tokens instead
// (two per warp, every row of the mma tile used): half the CTAs, and B[h] staged once per 16 tokens.  Instead of split partials the kernel
// can take num_parts reduced (z fp32 [T,H,W], lse [H,T]) pairs and LSE-merge them - how a
// sequence-split history arrives after its cross-GPU exchange.
#include "combine.cuh"
#include "common.cuh"
#include "decode_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

constexpr int kCTok = 8;       // tokens per CTA with the window inside (one per warp; the mma M of 16 is zero-padded)
constexpr int kCTokWide = 16;  // tokens per CTA with an external exact part (two per warp)
constexpr int kCKC = 64;       // k rows of B per chunk
constexpr int kCChunkBytes = kCKC * 128 * 2;   // 16 KB

template <int W, int TOK>
struct CombineSmem {
  static constexpr int Z_BYTES = 16 * W * 2;
  static constexpr int B_OFF = 0;                                // all of B[h]: W/64 chunks
  static constexpr int Z_OFF = (W / kCKC) * kCChunkBytes;
  static constexpr int OW_OFF = Z_OFF + Z_BYTES;                 // float [TOK][128] exact-part outputs
  static constexpr int Q_OFF = OW_OFF + TOK * 128 * 4;            // float [8 warps][128]
  static constexpr int L_OFF = Q_OFF + 8 * 128 * 4;               // float lse_h[TOK], lse_w[TOK]
  static constexpr int QSL_OFF = L_OFF + 2 * TOK * 4;           // int32 query_start_loc copy
  static constexpr int V_OFF = QSL_OFF + kQslCap * 4;            // per warp: the window's V rows
  // the 16-token form takes its exact part from outside and runs no window
  static constexpr int V_BYTES = TOK == kCTok ? 8 * kWindowVBytes : 0;
  static constexpr int BAR_OFF = V_OFF + V_BYTES;                // mbarrier: all of B[h] landed
  static constexpr int BYTES = BAR_OFF + 16 + 1024;              // + slack to align the base to 1024 B
};

template <int W, int TOK>
__global__ void __launch_bounds__(256, 1) decode_combine_kernel(const __grid_constant__ CUtensorMap tmap_b,
                                                             const CombineParams p) {
  static_assert(TOK == kCTok || TOK == kCTokWide, "8 or 16 tokens per CTA");
  using S = CombineSmem<W, TOK>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // B[h] arrives by TMA with SWIZZLE_128B, whose pattern follows address bits: 1024-byte aligned base
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* ow_s = reinterpret_cast<float*>(smem + S::OW_OFF);
  float* q_s = reinterpret_cast<float*>(smem + S::Q_OFF);
  float* lh_s = reinterpret_cast<float*>(smem + S::L_OFF);
  float* lw_s = lh_s + TOK;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, t0 = blockIdx.y * TOK, T = p.T, H = p.H;
  constexpr int NK = W / kCKC;

  // ---- all of B[h] in flight now (W/64 TMA boxes of 64 rows x 2 slabs of 64 columns, one mbarrier);
  //      it lands while steps 1-2 run.  Chunk kc holds [slab][row][64] with 128-byte rows swizzled
  //      by row % 8.
  uint64_t* bbar = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  if (tid == 0) {
    mbar_init(bbar, 1);
    fence_barrier_init();
    prefetch_tmap(&tmap_b);
    mbar_arrive_expect_tx(bbar, W * 128 * 2);
    for (int kc = 0; kc < NK; ++kc) tma_load_4d(smem + S::B_OFF + kc * kCChunkBytes, &tmap_b, bbar, 0, kc * kCKC, 0, h);
  }
  __syncthreads();  // the barrier is initialised before any thread waits on it
  WindowArgs win = p.win;
  win.qsl = stage_qsl(p.win.qsl, p.win.R, reinterpret_cast<int32_t*>(smem + S::QSL_OFF));

  // ---- 1 + 2: warp w owns tokens t0 + w (+ 8 in the 16-token form): exact window first (its inputs
  //      precede the history kernel), then - after the history grid has completed - the history reduce
#pragma unroll 1
  for (int tt = warp; tt < TOK; tt += 8) {
    const int t = t0 + tt;
    float o[4], lse_w;
    if (t < T && p.chunk_o) {
      const __nv_bfloat16* src = p.chunk_o + static_cast<int64_t>(t) * p.co_st + static_cast<int64_t>(h) * p.co_sh;
      const uint2 u = *reinterpret_cast<const uint2*>(src + lane * 4);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
      o[0] = __bfloat162float(b[0].x);
      o[1] = __bfloat162float(b[0].y);
      o[2] = __bfloat162float(b[1].x);
      o[3] = __bfloat162float(b[1].y);
      lse_w = p.chunk_lse[static_cast<int64_t>(h) * T + t];
    } else if (t < T && S::V_BYTES > 0) {
      if (!win.ctx_tok && win.window <= 32)
        window_warp_short(win, t, h, q_s + warp * 128, smem + S::V_OFF + warp * kWindowVBytes, o, lse_w);
      else window_warp(win, t, h, q_s + warp * 128, o, lse_w);
    } else {  // past T (the host launches the 16-token form only with an external exact part)
      o[0] = o[1] = o[2] = o[3] = 0.f;
      lse_w = -INFINITY;
    }
    griddep_wait();
    constexpr int NV = W / 128;  // float4 per lane
    float4 acc[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    float lse_h = -INFINITY;
    if (t < T && !(p.empty && p.empty[t])) {
      if (p.z_in) {
        // num_parts reduced partials (e.g. one per GPU of a sequence split): LSE-merge them
        float mx = -INFINITY;
        // L2-coherent loads (.cg): parts may have been stored by other GPUs during this kernel
        for (int q = 0; q < p.num_parts; ++q)
          mx = fmaxf(mx, __ldcg(p.lse_in + q * p.part_stride + static_cast<int64_t>(h) * T + t));
        if (mx != -INFINITY) {
          float wsum = 0.f;
          for (int q = 0; q < p.num_parts; ++q) {
            const float lq = __ldcg(p.lse_in + q * p.part_stride + static_cast<int64_t>(h) * T + t);
            if (lq == -INFINITY) continue;
            const float wgt = expf(lq - mx);
            wsum += wgt;
            const float4* src =
                reinterpret_cast<const float4*>(p.z_in + q * p.part_stride + (static_cast<int64_t>(t) * H + h) * W);
#pragma unroll
            for (int i = 0; i < NV; ++i) {
              const float4 v = __ldcg(src + i * 32 + lane);
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
      } else if (p.zw_in) {
        // num_parts parts as exchange words stored by the parts' GPUs (history_reduce_exchange): each
        // word is polled until it carries this exchange's tag.  The lse words (lane q polls part q's)
        // and the first two parts' z words in one memory round, then the z words of two parts per
        // round; the merge order is the one above.
        WordPoll poll(static_cast<uint32_t>(*p.epoch) + 1u, p.wait_ns);
        uint64_t wv[2][NV][4];
        const uint64_t* src[2];
        auto load_pair = [&](int u, int q) {
          src[u] = p.zw_in + q * p.part_stride + (static_cast<int64_t>(t) * H + h) * W;
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            ld_words2(src[u] + (i * 32 + lane) * 4, wv[u][i][0], wv[u][i][1]);
            ld_words2(src[u] + (i * 32 + lane) * 4 + 2, wv[u][i][2], wv[u][i][3]);
          }
        };
        // the first two parts' z words go out with the lse words (one memory round instead of two; a part
        // that turns out to have no keys has loaded for nothing)
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (u < p.num_parts) load_pair(u, u);
        float lq = -INFINITY;
        if (lane < p.num_parts) {
          const uint64_t* lsrc = p.lw_in + lane * p.part_stride + static_cast<int64_t>(h) * T + t;
          uint64_t w = ld_word(lsrc);
          if (poll.wait1(lsrc, w)) lq = word_value(w);
        }
        const float mx = warp_max(lq);
        if (mx != -INFINITY) {
          float wsum = 0.f;
          for (int q0 = 0; q0 < p.num_parts; q0 += 2) {
            float lu[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int q = q0 + u;
              lu[u] = __shfl_sync(0xffffffffu, lq, q < p.num_parts ? q : 0);
              if (q >= p.num_parts) lu[u] = -INFINITY;
              if (q0 > 0 && lu[u] != -INFINITY) load_pair(u, q);  // pair 0 is already in flight
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (lu[u] == -INFINITY) continue;  // past the parts, or a part without keys
              const float wgt = expf(lu[u] - mx);
              wsum += wgt;
#pragma unroll
              for (int i = 0; i < NV; ++i) {
                // words that never arrived count as zeros (after a timeout, words already there are taken)
                bool ok = poll.wait2(src[u] + (i * 32 + lane) * 4, wv[u][i][0], wv[u][i][1]);
                ok = poll.wait2(src[u] + (i * 32 + lane) * 4 + 2, wv[u][i][2], wv[u][i][3]) && ok;
                if (!ok) continue;
                acc[i].x += wgt * word_value(wv[u][i][0]); acc[i].y += wgt * word_value(wv[u][i][1]);
                acc[i].z += wgt * word_value(wv[u][i][2]); acc[i].w += wgt * word_value(wv[u][i][3]);
              }
            }
          }
          const float inv = 1.f / wsum;
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            acc[i].x *= inv; acc[i].y *= inv; acc[i].z *= inv; acc[i].w *= inv;
          }
          lse_h = mx + logf(wsum);
        }
        if (poll.failed) record_error(p.err, kErrWaitPeer);
      } else {
        int lo = t, hi = t + 1;
        if (p.stream_mode) {
          const int2 m = p.meta[t];
          lo = m.x;
          hi = m.y;
        }
        // up to 4 partial slots per pass, their lse and rows loaded together (one memory round for a row
        // with <= 4 partials); the running max rescales the sums when a later pass raises it
        float mx = -INFINITY, wsum = 0.f;
        for (int s0 = lo; s0 < hi; s0 += 4) {
          float ls[4];
          float4 v[4][NV];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int s = s0 + u;
            ls[u] = s < hi ? p.ws_lse[static_cast<int64_t>(s) * H + h] : -INFINITY;
            const float4* src = reinterpret_cast<const float4*>(p.ws_o + (static_cast<int64_t>(s < hi ? s : lo) * H + h) * W);
#pragma unroll
            for (int i = 0; i < NV; ++i) v[u][i] = s < hi ? src[i * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          const float m2 = fmaxf(fmaxf(mx, fmaxf(ls[0], ls[1])), fmaxf(ls[2], ls[3]));
          if (m2 == -INFINITY) continue;
          if (m2 != mx) {
            const float sc = expf(mx - m2);  // 0 while nothing has been summed (mx = -inf)
            wsum *= sc;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
              acc[i].x *= sc; acc[i].y *= sc; acc[i].z *= sc; acc[i].w *= sc;
            }
            mx = m2;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (ls[u] == -INFINITY) continue;  // past hi, or a slot without keys
            const float wgt = expf(ls[u] - mx);
            wsum += wgt;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
              acc[i].x += wgt * v[u][i].x; acc[i].y += wgt * v[u][i].y;
              acc[i].z += wgt * v[u][i].z; acc[i].w += wgt * v[u][i].w;
            }
          }
        }
        if (mx != -INFINITY) {
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
    for (int i = 0; i < NV; ++i) {  // z row tt: dims 4(32i + lane) .. +3 as bf16 into the swizzled tile
      const int d = (i * 32 + lane) * 4;
      uint2 pk;
      pk.x = pack_bf16(acc[i].x, acc[i].y);
      pk.y = pack_bf16(acc[i].z, acc[i].w);
      *reinterpret_cast<uint2*>(smem + S::Z_OFF + swz(tt, d >> 3, W * 2) + (d & 7) * 2) = pk;
      if (TOK == kCTok)  // 8 tokens: rows 8-15 of the mma tile are zero
        *reinterpret_cast<uint2*>(smem + S::Z_OFF + swz(tt + 8, d >> 3, W * 2) + (d & 7) * 2) = make_uint2(0u, 0u);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) ow_s[tt * 128 + lane * 4 + e] = bf16_round(o[e]);
    if (lane == 0) {
      lh_s[tt] = lse_h;
      lw_s[tt] = lse_w;
    }
  }

  // ---- 3: o_hist[16 x 128] = z[16 x W] . B[h][W x 128]; warp w owns columns 16w .. 16w+15
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const uint32_t zb = smem_u32(smem + S::Z_OFF);
  if (!mbar_wait(bbar, 0, p.wait_ns)) record_error(p.err, kErrWaitFull);
  __syncthreads();
  if (p.epoch && tid == 0) {
    // every warp of this CTA has taken its exchange words (the z tile is complete); the last CTA
    // through advances the slot's use counter, so the slot's next exchange carries a new tag
    const unsigned total = gridDim.x * gridDim.y;
    if (atom_add_acq_rel_gpu(reinterpret_cast<unsigned*>(p.part_seen), 1u) == total - 1) {
      *p.epoch += 1;
      *p.part_seen = 0;
    }
  }
  for (int kc = 0; kc < NK; ++kc) {
    const uint32_t bb = smem_u32(smem + S::B_OFF + kc * kCChunkBytes);
#pragma unroll
    for (int ks = 0; ks < kCKC / 16; ++ks) {
      uint32_t a[4], b0, b1, b2, b3;
      const int arow = (lane & 7) + ((lane >> 3) & 1) * 8;
      ldsm_x4(zb + swz(arow, (kc * kCKC + ks * 16) / 8 + (lane >> 4), W * 2), a[0], a[1], a[2], a[3]);
      const int krow = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int bch = 2 * warp + (lane >> 4);  // 16-byte chunk of the 128 columns: slab bch / 8
      ldsm_x4_t(bb + (bch >> 3) * (kCKC * 128) + krow * 128 + ((((bch & 7) ^ (krow & 7))) << 4), b0, b1, b2, b3);
      mma_bf16_16816(acc[0], a, b0, b1);
      mma_bf16_16816(acc[1], a, b2, b3);
    }
  }

  // ---- 4: merge (row g (+ 8) of the mma tile = token t0 + g (+ 8); columns 16w + 8nt + 2c, +1)
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int half = 0; half < TOK / 8; ++half) {
    const int tt = g + 8 * half, t = t0 + tt;
    if (t >= T) return;
    const bool invalid = t >= win.qsl[win.R];
    float w1, w2;
    merge_weights_states(lh_s[tt], lw_s[tt], w1, w2);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int col = 16 * warp + 8 * nt + 2 * c;
      float r0 = bf16_round(acc[nt][2 * half]) * w1 + ow_s[tt * 128 + col] * w2;
      float r1 = bf16_round(acc[nt][2 * half + 1]) * w1 + ow_s[tt * 128 + col + 1] * w2;
      if (invalid) r0 = r1 = 0.f;
      *reinterpret_cast<__nv_bfloat162*>(p.out + static_cast<int64_t>(t) * p.o_st + static_cast<int64_t>(h) * p.o_sh +
                                         col) = __floats2bfloat162_rn(r0, r1);
    }
    if (warp == 0 && c == 0 && p.lse_out)
      p.lse_out[static_cast<int64_t>(h) * T + t] = invalid ? -INFINITY : merged_lse(lh_s[tt], lw_s[tt]);
  }
}

template <int W, int TOK>
static int launch_combine(const CombineParams& p, bool pdl, cudaStream_t s) {
  CUtensorMap tb;
  int rc = combine_b_tmap(&tb, p.B, p.H, W, p.b_sh, p.b_sk);
  if (rc) return rc;
  static unsigned attr_mask = 0;
  const int smem = CombineSmem<W, TOK>::BYTES;
  ensure_smem_limit(decode_combine_kernel<W, TOK>, smem, attr_mask);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.H, (p.T + TOK - 1) / TOK);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, decode_combine_kernel<W, TOK>, tb, p), "decode_combine_kernel launch");
}

// The 16-token form when the exact part comes from outside and the 8-token grid would not fit in one
// wave (one CTA per SM: its shared memory holds all of B[h])
static bool combine_wide(const CombineParams& p) {
  if (!p.chunk_o) return false;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return false;
  return static_cast<int64_t>(p.H) * ((p.T + kCTok - 1) / kCTok) > sms;
}

int decode_combine(const CombineParams& p, int W, bool pdl, cudaStream_t s) {
  if (p.T == 0) return kStatusOk;
  const bool wide = combine_wide(p);
  switch (W) {
    case 256: return wide ? launch_combine<256, kCTokWide>(p, pdl, s) : launch_combine<256, kCTok>(p, pdl, s);
    case 512: return wide ? launch_combine<512, kCTokWide>(p, pdl, s) : launch_combine<512, kCTok>(p, pdl, s);
    default: set_error("decode combine width %d unsupported (256 or 512)", W); return kStatusInvalid;
  }
}

}  // namespace hla
