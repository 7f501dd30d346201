// Device helpers and argument blocks shared by decode_ops.cu and combine.cu.
#pragma once
#include "common.cuh"

namespace hla {

__device__ __forceinline__ int64_t clamp_pos(int64_t p, int64_t max_pos) {
  return p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);
}

// Token -> request of a varlen batch (s6_ops.py:61-68): r = #{i in 1..R : qsl[i] <= t},
// clamped to R - 1; valid = t < qsl[R].
__device__ __forceinline__ bool token_request(const int32_t* __restrict__ qsl, int R, int t, int& r) {
  int lo = 1, hi = R + 1;  // first i in [1, R] with qsl[i] > t
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (qsl[mid] <= t) lo = mid + 1; else hi = mid;
  }
  r = min(lo - 1, R - 1);
  return t < qsl[R];
}

// Copy query_start_loc [R + 1] into shared memory (all threads of the CTA must call this) so the
// per-token binary searches run on shared memory; falls back to the global array when it does
// not fit in `cap` entries.
constexpr int kQslCap = 1024;
__device__ __forceinline__ const int32_t* stage_qsl(const int32_t* __restrict__ qsl, int R, int32_t* buf) {
  if (R + 1 > kQslCap) return qsl;
  for (int i = threadIdx.x; i <= R; i += blockDim.x) buf[i] = qsl[i];
  __syncthreads();
  return buf;
}

// vLLM slot of token t at position pos: block_table[req, pos / page] * page + pos % page, or -1 for a
// padding token, a negative position, a column past the table or a block id outside the cache.
__device__ __forceinline__ int64_t token_slot(const int32_t* qsl, int R, int t, int64_t pos, const int32_t* bt,
                                              int64_t bt_st, int max_blocks, int page, int64_t num_blocks) {
  int r;
  if (!token_request(qsl, R, t, r) || pos < 0) return -1;
  const int64_t col = pos / page;
  if (col >= max_blocks) return -1;
  const int blk = bt[static_cast<int64_t>(r) * bt_st + col];
  if (blk < 0 || blk >= num_blocks) return -1;
  return static_cast<int64_t>(blk) * page + pos % page;
}

// Neox rotate-half pair (x1 at i, x2 at i + w/2) in the torch bf16 operation order:
// y1 = bf16(bf16(x1*c) + bf16(-x2*s)), y2 = bf16(bf16(x2*c) + bf16(x1*s)).
__device__ __forceinline__ void rope_pair_torch(float x1, float x2, float c, float s, float& y1, float& y2) {
  const float a1 = bf16_round(x1 * c), b1 = bf16_round(-x2 * s);
  const float a2 = bf16_round(x2 * c), b2 = bf16_round(x1 * s);
  y1 = bf16_round(a1 + b1);
  y2 = bf16_round(a2 + b2);
}

// merge_states weights (s6_ops.py:275-284): +inf lse is empty, both empty -> 0.
__device__ __forceinline__ void merge_weights_states(float l1, float l2, float& w1, float& w2) {
  if (l1 == INFINITY) l1 = -INFINITY;
  if (l2 == INFINITY) l2 = -INFINITY;
  float peak = fmaxf(l1, l2);
  if (isinf(peak)) peak = 0.f;
  const float e1 = expf(l1 - peak), e2 = expf(l2 - peak), tot = e1 + e2;
  w1 = tot > 0.f ? e1 / tot : 0.f;
  w2 = tot > 0.f ? e2 / tot : 0.f;
}

// merge_lse weights (s6_ops.py:353-361).
__device__ __forceinline__ void merge_weights_lse(float l1, float l2, float& w1, float& w2) {
  float peak = fmaxf(l1, l2);
  if (isinf(peak)) peak = 0.f;
  const float e1 = expf(l1 - peak), e2 = expf(l2 - peak), tot = e1 + e2;
  w1 = tot > 0.f ? e1 / tot : 0.f;
  w2 = tot > 0.f ? e2 / tot : 0.f;
}

__device__ __forceinline__ float merged_lse(float l1, float l2) {
  float peak = fmaxf(l1, l2);
  if (isinf(peak)) peak = 0.f;
  return peak + logf(expf(l1 - peak) + expf(l2 - peak));
}

// ------------------------------------------------------------------ exact window (A5)
struct WindowArgs {
  const __nv_bfloat16* q;  // roped q [T, H, 128]
  int64_t q_st, q_sh;
  const __nv_bfloat16* cache;  // logical [nb, H, page, 256] (K | V); strides per block, head, row
  int64_t c_sb, c_sh, c_sr;
  int64_t num_blocks;
  int page;
  const int32_t* bt;  // per-request block table [R, max_blocks]
  int64_t bt_st;
  int max_blocks;
  const int32_t* qsl;  // query_start_loc [R + 1]
  int R;
  const int32_t* seq_lens;  // [R]
  int window;
  float scale;
  // per-token history mode (window_history_fa): when set, token t reads rows [ctx_tok[t] - window,
  // ctx_tok[t]) through row t of a per-token block table, without the current token
  const int32_t* ctx_tok;
};

// One warp computes the exact window attention of token t, head h over keys
// [pos - window, pos] (pos = seq_len - query_len + index in chunk; for decode seq_len - 1),
// the current token included.  Lane l scores keys l, l + 32, ... (its K row is read with 16
// independent 16-byte loads), then owns output dims 4l..4l+3 and accumulates V in groups of 16
// keys whose loads are issued together.  Invalid tokens or an empty key range give o = 0,
// lse = -inf.  q_s: 128 floats of this warp's shared memory.
__device__ __forceinline__ void window_warp(const WindowArgs& a, int t, int h, float* q_s, float (&o)[4],
                                            float& lse) {
  const int lane = threadIdx.x & 31;
  o[0] = o[1] = o[2] = o[3] = 0.f;
  lse = -INFINITY;
  int r, win = a.window;
  int64_t pos;
  if (a.ctx_tok) {
    r = t;
    pos = static_cast<int64_t>(a.ctx_tok[t]) - 1;
    win = a.window - 1;
    if (a.window <= 0) return;
  } else {
    if (!token_request(a.qsl, a.R, t, r)) return;
    const int qlen = a.qsl[r + 1] - a.qsl[r];
    pos = static_cast<int64_t>(a.seq_lens[r]) - qlen + (t - a.qsl[r]);
  }
  if (pos < 0) return;
  const int64_t first = pos - win > 0 ? pos - win : 0;
  const int n = static_cast<int>(pos - first + 1);
  {
    const __nv_bfloat16* qp = a.q + static_cast<int64_t>(t) * a.q_st + static_cast<int64_t>(h) * a.q_sh + lane * 4;
    const uint2 u = *reinterpret_cast<const uint2*>(qp);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
    __syncwarp();
    q_s[lane * 4 + 0] = __bfloat162float(b[0].x);
    q_s[lane * 4 + 1] = __bfloat162float(b[0].y);
    q_s[lane * 4 + 2] = __bfloat162float(b[1].x);
    q_s[lane * 4 + 3] = __bfloat162float(b[1].y);
  }
  __syncwarp();
  constexpr int MAXC = 4;  // up to 128 keys (window <= 127)
  float sc[MAXC];
  int64_t off[MAXC];
  float mx = -INFINITY;
#pragma unroll
  for (int ch = 0; ch < MAXC; ++ch) {
    sc[ch] = -INFINITY;
    off[ch] = -1;
    if (ch * 32 >= n) continue;
    const int kb = ch * 32 + lane;
    if (kb < n) {
      const int64_t j = first + kb;
      const int64_t col = j / a.page;
      if (col < a.max_blocks) {
        const int blk = a.bt[static_cast<int64_t>(r) * a.bt_st + col];
        if (blk >= 0 && blk < a.num_blocks)
          off[ch] = static_cast<int64_t>(blk) * a.c_sb + static_cast<int64_t>(h) * a.c_sh + (j % a.page) * a.c_sr;
      }
    }
    if (off[ch] >= 0) {
      const uint4* kp = reinterpret_cast<const uint4*>(a.cache + off[ch]);
      uint4 kr[16];
#pragma unroll
      for (int v = 0; v < 16; ++v) kr[v] = __ldg(kp + v);
      float dot = 0.f;
#pragma unroll
      for (int v = 0; v < 16; ++v) {
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&kr[v]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          dot = fmaf(q_s[v * 8 + 2 * e], __bfloat162float(b[e].x), dot);
          dot = fmaf(q_s[v * 8 + 2 * e + 1], __bfloat162float(b[e].y), dot);
        }
      }
      sc[ch] = dot * a.scale;
    }
    mx = fmaxf(mx, sc[ch]);
  }
  mx = warp_max(mx);
  if (mx == -INFINITY) return;
  float l = 0.f;
#pragma unroll
  for (int ch = 0; ch < MAXC; ++ch) {
    sc[ch] = sc[ch] == -INFINITY ? 0.f : expf(sc[ch] - mx);
    l += sc[ch];
  }
  l = warp_sum(l);
#pragma unroll
  for (int ch = 0; ch < MAXC; ++ch) {
    if (ch * 32 >= n) break;
#pragma unroll
    for (int g0 = 0; g0 < 32; g0 += 16) {
      if (ch * 32 + g0 >= n) break;
      float pw[16];
      uint2 vv[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        pw[e] = __shfl_sync(0xffffffffu, sc[ch], g0 + e);
        const int64_t ro = __shfl_sync(0xffffffffu, off[ch], g0 + e);
        const bool live = (ch * 32 + g0 + e < n) && ro >= 0;
        vv[e] = live ? __ldg(reinterpret_cast<const uint2*>(a.cache + ro + 128 + lane * 4)) : make_uint2(0u, 0u);
        if (!live) pw[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&vv[e]);
        o[0] = fmaf(pw[e], __bfloat162float(b[0].x), o[0]);
        o[1] = fmaf(pw[e], __bfloat162float(b[0].y), o[1]);
        o[2] = fmaf(pw[e], __bfloat162float(b[1].x), o[2]);
        o[3] = fmaf(pw[e], __bfloat162float(b[1].y), o[3]);
      }
    }
  }
  const float inv = 1.f / l;
  o[0] *= inv;
  o[1] *= inv;
  o[2] *= inv;
  o[3] *= inv;
  lse = mx + logf(l);
}

// window_warp for a window of at most 32 history keys (the decode window, W = 32) in two dependent
// memory rounds instead of one per 16 keys: round 1 fetches q and the block-table entries of every
// key, round 2 puts every K and V load in flight at once - lane l's K row (history key first + l)
// into registers and its V row into this warp's shared buffer with cp.async, so the 32 V rows take
// no registers (held in registers they outgrew what the compiler keeps in flight, and the loads
// went out in several rounds).  The value accumulation then reads its 4 dims of every key's V row
// from shared memory.  A 33rd key (the current token when the window is full) is scored by the
// whole warp (4 dims per lane, warp sum).  Same math and key order as window_warp.  Only for the
// decode mode (ctx_tok unset) with window <= 32.  v_s: kWindowVBytes of this warp's shared memory,
// 16-byte aligned; rows are stored with their 16-byte chunks XOR-swizzled by key % 16.
constexpr int kWindowVBytes = 32 * 256;
__device__ __forceinline__ void window_warp_short(const WindowArgs& a, int t, int h, float* q_s, uint8_t* v_s,
                                                  float (&o)[4], float& lse) {
  const int lane = threadIdx.x & 31;
  o[0] = o[1] = o[2] = o[3] = 0.f;
  lse = -INFINITY;
  int r;
  if (!token_request(a.qsl, a.R, t, r)) return;
  const int qlen = a.qsl[r + 1] - a.qsl[r];
  const int64_t pos = static_cast<int64_t>(a.seq_lens[r]) - qlen + (t - a.qsl[r]);
  if (pos < 0) return;
  const int64_t first = pos - a.window > 0 ? pos - a.window : 0;
  const int n = static_cast<int>(pos - first + 1);          // <= 33
  const int nl = n < 32 ? n : 32;                           // keys owned by lanes; key 32 (if any) is shared
  auto row_of = [&](int64_t j) -> int64_t {                 // element offset of key j's row, or -1
    const int64_t col = j / a.page;
    if (col >= a.max_blocks) return -1;
    const int blk = a.bt[static_cast<int64_t>(r) * a.bt_st + col];
    if (blk < 0 || blk >= a.num_blocks) return -1;
    return static_cast<int64_t>(blk) * a.c_sb + static_cast<int64_t>(h) * a.c_sh + (j % a.page) * a.c_sr;
  };
  // ---- round 1: q and the rows' block ids
  const uint2 qu = *reinterpret_cast<const uint2*>(a.q + static_cast<int64_t>(t) * a.q_st +
                                                   static_cast<int64_t>(h) * a.q_sh + lane * 4);
  const int64_t off = lane < nl ? row_of(first + lane) : -1;
  const int64_t offx = n > 32 ? row_of(first + 32) : -1;   // same address in every lane
  {
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&qu);
    __syncwarp();
    q_s[lane * 4 + 0] = __bfloat162float(b[0].x);
    q_s[lane * 4 + 1] = __bfloat162float(b[0].y);
    q_s[lane * 4 + 2] = __bfloat162float(b[1].x);
    q_s[lane * 4 + 3] = __bfloat162float(b[1].y);
  }
  __syncwarp();
  // ---- round 2: every K and V load of the window.  V row of key l -> v_s + 256 l (zeros for a key
  //      without a row), chunk c at chunk position c ^ (l % 16)
  {
    const __nv_bfloat16* vrow = a.cache + (off >= 0 ? off : 0) + 128;
#pragma unroll
    for (int c = 0; c < 16; ++c) cp_async16(v_s + lane * 256 + ((c ^ (lane & 15)) << 4), vrow + c * 8, off >= 0 ? 16 : 0);
    cp_async_commit();
  }
  uint4 kr[16];
  if (off >= 0) {
    const uint4* kp = reinterpret_cast<const uint4*>(a.cache + off);
#pragma unroll
    for (int v = 0; v < 16; ++v) kr[v] = __ldg(kp + v);
  }
  uint2 kx = make_uint2(0u, 0u), vx = make_uint2(0u, 0u);
  if (offx >= 0) {
    kx = __ldg(reinterpret_cast<const uint2*>(a.cache + offx + lane * 4));
    vx = __ldg(reinterpret_cast<const uint2*>(a.cache + offx + 128 + lane * 4));
  }
  // ---- scores
  float sc = -INFINITY;
  if (off >= 0) {
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < 16; ++v) {
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&kr[v]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dot = fmaf(q_s[v * 8 + 2 * e], __bfloat162float(b[e].x), dot);
        dot = fmaf(q_s[v * 8 + 2 * e + 1], __bfloat162float(b[e].y), dot);
      }
    }
    sc = dot * a.scale;
  }
  float scx = -INFINITY;
  if (offx >= 0) {
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&kx);
    float part = q_s[lane * 4 + 0] * __bfloat162float(b[0].x);
    part = fmaf(q_s[lane * 4 + 1], __bfloat162float(b[0].y), part);
    part = fmaf(q_s[lane * 4 + 2], __bfloat162float(b[1].x), part);
    part = fmaf(q_s[lane * 4 + 3], __bfloat162float(b[1].y), part);
    scx = warp_sum(part) * a.scale;
  }
  cp_async_wait<0>();  // this lane's V row has landed
  __syncwarp();        // ... and every other lane's
  const float mx = fmaxf(warp_max(sc), scx);
  if (mx == -INFINITY) return;
  const float p = sc == -INFINITY ? 0.f : expf(sc - mx);
  const float px = scx == -INFINITY ? 0.f : expf(scx - mx);
  const float l = warp_sum(p) + px;
  const int vchunk = lane >> 1, vhalf = (lane & 1) * 8;  // dims 4 lane .. + 3 of a V row
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const float pw = __shfl_sync(0xffffffffu, p, e);
    const uint2 vv = *reinterpret_cast<const uint2*>(v_s + e * 256 + ((vchunk ^ (e & 15)) << 4) + vhalf);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&vv);
    o[0] = fmaf(pw, __bfloat162float(b[0].x), o[0]);
    o[1] = fmaf(pw, __bfloat162float(b[0].y), o[1]);
    o[2] = fmaf(pw, __bfloat162float(b[1].x), o[2]);
    o[3] = fmaf(pw, __bfloat162float(b[1].y), o[3]);
  }
  {
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&vx);
    o[0] = fmaf(px, __bfloat162float(b[0].x), o[0]);
    o[1] = fmaf(px, __bfloat162float(b[0].y), o[1]);
    o[2] = fmaf(px, __bfloat162float(b[1].x), o[2]);
    o[3] = fmaf(px, __bfloat162float(b[1].y), o[3]);
  }
  const float inv = 1.f / l;
  o[0] *= inv;
  o[1] *= inv;
  o[2] *= inv;
  o[3] *= inv;
  lse = mx + logf(l);
}

// ------------------------------------------------------------------ exact append (A10)
struct ExactArgs {
  __nv_bfloat16* q;  // [T, H, 128] roped in place (may be NULL)
  int64_t q_st, q_sh;
  const __nv_bfloat16* k;
  int64_t k_st, k_sh;
  const __nv_bfloat16* v;
  int64_t v_st, v_sh;
  __nv_bfloat16* k_out;  // optional roped k copy [T, H, 128]
  int64_t ko_st, ko_sh;
  const int64_t* positions;
  const float* cos_sin;  // [max_pos, 128] = [cos 64 | sin 64] fp32
  int64_t cs_st, max_pos;
  __nv_bfloat16* cache;  // logical [nb, H, page, 256]
  int64_t c_sb, c_sh, c_sr, num_blocks;
  int page;
  const int32_t* bt;
  int64_t bt_st;
  int max_blocks;
  const int32_t* qsl;
  int R, H;
  int64_t* slot_out;  // optional [T]
};

// ------------------------------------------------------------------ committed rows (A9 + A10)
struct CommitArgs {
  const __nv_bfloat16* row;  // [T, 2w] (K | V)
  int64_t row_st;
  int w;
  const int64_t* positions;
  const __nv_bfloat16* table;  // [max_pos, w] = [cos | sin]
  int64_t tab_st, max_pos;
  __nv_bfloat16* cache;  // [nb, 1, page, 2w]
  int64_t c_sb, c_sr, num_blocks;
  int page;
  const int32_t* bt;  // per-request block table
  int64_t bt_st;
  int max_blocks;
  const int32_t* qsl;
  int R;
  int64_t* slot_out;
};

// host launchers (decode_ops.cu)
int window_attention(const WindowArgs& a, int T, int H, void* out, int64_t o_st, int64_t o_sh, float* lse,
                     cudaStream_t s);
int merge(const void* o1, int64_t s1t, int64_t s1h, const float* lse1, const void* o2, int64_t s2t, int64_t s2h,
          const float* lse2, const uint8_t* invalid, void* out, int64_t sot, int64_t soh, float* lse_out, int T, int H,
          int D, int mode, cudaStream_t s);
int latent_rope(void* x, int64_t st, int64_t sh, int T, int H, int w, const int64_t* positions, const void* table,
                int64_t tab_st, int64_t max_pos, cudaStream_t s);
int exact_append(const ExactArgs& a, int T, cudaStream_t s);
int commit_rows(const CommitArgs& a, int T, cudaStream_t s);

}  // namespace hla
