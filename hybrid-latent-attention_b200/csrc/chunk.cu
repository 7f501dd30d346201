// Causal attention inside each request's current chunk (reference s6_ops.py:234-259,
// chunk_attention: FA2 varlen causal over cu_seqlens = query_start_loc; torch oracle
// _chunk_reference).  Token i attends to tokens j <= i of its own request.  Padding tokens
// (i >= query_start_loc[R]) give o = 0 and lse = -inf.
//
// FlashAttention-2 style on mma.m16n8k16: a CTA owns 64 query tokens of one head (4 warps x 16
// rows), Q stays in registers, K and V tiles of 64 keys stream through a cp.async double buffer in
// XOR-swizzled shared memory, scores are masked by (same request, causal), softmax is online in
// the log2 domain and P is reused from the score fragments for P.V.
#include "common.cuh"
#include "decode_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

struct ChunkParams {
  const __nv_bfloat16 *q, *k, *v;  // [T, H, 128]
  int64_t q_st, q_sh, k_st, k_sh, v_st, v_sh;
  const int32_t* qsl;
  int R, T, H;
  float scale_log2;
  __nv_bfloat16* out;  // [T, H, 128]
  int64_t o_st, o_sh;
  float* lse;  // [H, T]
};

constexpr int kChTile = 64;
constexpr int kChTileBytes = kChTile * 256;  // 64 rows x 128 bf16

__global__ void __launch_bounds__(128) chunk_attn_kernel(const ChunkParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* qs = smem;                                // [64][256 B]
  uint8_t* ks = smem + kChTileBytes;                 // 2 x [64][256 B]
  uint8_t* vs = smem + 3 * kChTileBytes;             // 2 x [64][256 B]
  int32_t* rq = reinterpret_cast<int32_t*>(smem + 5 * kChTileBytes);  // request of each query row
  int32_t* rk = rq + kChTile;                                        // 2 x request of each key
  int32_t* qsl_s = rk + 2 * kChTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int t0 = blockIdx.x * kChTile, h = blockIdx.y, T = p.T;
  const int32_t* qsl = stage_qsl(p.qsl, p.R, qsl_s);
  const int total = qsl[p.R];  // valid tokens

  for (int i = tid; i < kChTile; i += blockDim.x) {
    int r = -1;
    if (t0 + i < T && t0 + i < total) token_request(qsl, p.R, t0 + i, r);
    rq[i] = r;
  }
  __syncthreads();
  // key range: from the start of the first valid row's request to the last row
  const int kmin = (rq[0] >= 0) ? qsl[rq[0]] : t0;
  const int kmax = min(min(t0 + kChTile, T), total) - 1;  // inclusive
  const int ntiles = kmax >= kmin ? (kmax - kmin) / kChTile + 1 : 0;

  auto load_kv = [&](int buf, int j0) {
    for (int idx = tid; idx < kChTile * 16; idx += blockDim.x) {
      const int row = idx >> 4, ch = idx & 15, j = j0 + row;
      const bool in = j <= kmax;
      const int jj = in ? j : kmin;
      cp_async16(ks + buf * kChTileBytes + swz(row, ch, 256),
                 p.k + static_cast<int64_t>(jj) * p.k_st + static_cast<int64_t>(h) * p.k_sh + ch * 8, in ? 16 : 0);
      cp_async16(vs + buf * kChTileBytes + swz(row, ch, 256),
                 p.v + static_cast<int64_t>(jj) * p.v_st + static_cast<int64_t>(h) * p.v_sh + ch * 8, in ? 16 : 0);
    }
    for (int i = tid; i < kChTile; i += blockDim.x) {
      const int j = j0 + i;
      int r = -1;
      if (j <= kmax) token_request(qsl, p.R, j, r);
      rk[buf * kChTile + i] = r;
    }
  };
  // Q tile
  for (int idx = tid; idx < kChTile * 16; idx += blockDim.x) {
    const int row = idx >> 4, ch = idx & 15, t = t0 + row;
    const bool in = t < T;
    cp_async16(qs + swz(row, ch, 256),
               p.q + static_cast<int64_t>(in ? t : 0) * p.q_st + static_cast<int64_t>(h) * p.q_sh + ch * 8,
               in ? 16 : 0);
  }
  if (ntiles > 0) load_kv(0, kmin);
  cp_async_commit();

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  uint32_t qa[8][4];
  const int row0 = warp * 16 + g, row1 = row0 + 8;  // tile rows of this thread
  const int i0 = t0 + row0, i1 = t0 + row1;         // their token indices

  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1, j0 = kmin + it * kChTile;
    if (it + 1 < ntiles) load_kv(buf ^ 1, j0 + kChTile);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (it == 0) {
      const uint32_t qb = smem_u32(qs);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int arow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm_x4(qb + swz(arow, kk * 2 + (lane >> 4), 256), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
      }
    }
    const uint32_t kb = smem_u32(ks + buf * kChTileBytes), vb = smem_u32(vs + buf * kChTileBytes);
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
      const int key = jp * 16 + ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz(key, kk * 2 + ((lane >> 3) & 1), 256), b0, b1, b2, b3);
        mma_bf16_16816(sc[2 * jp], qa[kk], b0, b1);
        mma_bf16_16816(sc[2 * jp + 1], qa[kk], b2, b3);
      }
    }
    // mask: same request and causal; out-of-range keys have request -1
    const int rq0 = rq[row0], rq1 = rq[row1];
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kc = j * 8 + 2 * c + e, kj = j0 + kc, rkj = rk[buf * kChTile + kc];
        const bool ok0 = rq0 >= 0 && rkj == rq0 && kj <= i0;
        const bool ok1 = rq1 >= 0 && rkj == rq1 && kj <= i1;
        sc[j][e] = ok0 ? sc[j][e] * p.scale_log2 : -INFINITY;
        sc[j][2 + e] = ok1 ? sc[j][2 + e] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, sc[j][e]);
        mx1 = fmaxf(mx1, sc[j][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0, base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m_run[0] - base0), al1 = exp2f(m_run[1] - base1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e0 = exp2f(sc[j][0] - base0), e1 = exp2f(sc[j][1] - base0);
      const float e2 = exp2f(sc[j][2] - base1), e3 = exp2f(sc[j][3] - base1);
      rs0 += e0 + e1;
      rs1 += e2 + e3;
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16(e0, e1);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16(e2, e3);
    }
    l_run[0] = l_run[0] * al0 + rs0;
    l_run[1] = l_run[1] * al1 + rs1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= al0; o[j][1] *= al0;
      o[j][2] *= al1; o[j][3] *= al1;
    }
#pragma unroll
    for (int ks4 = 0; ks4 < 4; ++ks4) {
      const int key = ks4 * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
      for (int jd = 0; jd < 8; ++jd) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + swz(key, jd * 2 + (lane >> 4), 256), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * jd], pa[ks4], b0, b1);
        mma_bf16_16816(o[2 * jd + 1], pa[ks4], b2, b3);
      }
    }
    __syncthreads();  // this buffer is refilled by the next iteration's prefetch
  }
  cp_async_wait<0>();

  float l0 = l_run[0], l1 = l_run[1];
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float ln2 = 0.6931471805599453f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int t = half ? i1 : i0;
    if (t >= T) continue;
    const bool valid = (half ? rq[row1] : rq[row0]) >= 0;
    const float l = half ? l1 : l0;
    const float inv = (valid && l > 0.f) ? 1.f / l : 0.f;
    __nv_bfloat16* dst = p.out + static_cast<int64_t>(t) * p.o_st + static_cast<int64_t>(h) * p.o_sh;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = j * 8 + 2 * c;
      *reinterpret_cast<__nv_bfloat162*>(dst + d) =
          __floats2bfloat162_rn(o[j][2 * half] * inv, o[j][2 * half + 1] * inv);
    }
    if (c == 0) {
      const float m = half ? m_run[1] : m_run[0];
      p.lse[static_cast<int64_t>(h) * T + t] = (valid && l > 0.f) ? (m + log2f(l)) * ln2 : -INFINITY;
    }
  }
}

int chunk_attention(const ChunkParams& p, cudaStream_t s) {
  if (p.T == 0) return kStatusOk;
  const int smem = 5 * kChTileBytes + 3 * kChTile * 4 + kQslCap * 4;
  static unsigned attr_mask = 0;
  ensure_smem_limit(chunk_attn_kernel, smem, attr_mask);
  dim3 grid((p.T + kChTile - 1) / kChTile, p.H);
  chunk_attn_kernel<<<grid, 128, smem, s>>>(p);
  return cuda_status(cudaGetLastError(), "chunk_attn_kernel launch");
}

}  // namespace hla

using namespace hla;

extern "C" int hla_s6_chunk_attention(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                                      int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                                      int64_t v_stride_h, const int32_t* query_start_loc, int32_t num_reqs,
                                      int32_t num_tokens, int32_t num_heads, int32_t head_dim, float scale, void* out,
                                      int64_t out_stride_t, int64_t out_stride_h, float* lse, void* stream) {
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0; };
  if (head_dim != 128 || num_reqs < 1 || !al16(q) || !al16(k) || !al16(v) || (q_stride_t % 8) || (q_stride_h % 8) ||
      (k_stride_t % 8) || (k_stride_h % 8) || (v_stride_t % 8) || (v_stride_h % 8) || (out_stride_t % 2) ||
      (out_stride_h % 2)) {
    set_error("chunk attention needs head_dim 128, >= 1 request and 16-byte aligned q/k/v rows");
    return kStatusInvalid;
  }
  ChunkParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.k_st = k_stride_t;
  p.k_sh = k_stride_h;
  p.v_st = v_stride_t;
  p.v_sh = v_stride_h;
  p.qsl = query_start_loc;
  p.R = num_reqs;
  p.T = num_tokens;
  p.H = num_heads;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_st = out_stride_t;
  p.o_sh = out_stride_h;
  p.lse = lse;
  return chunk_attention(p, static_cast<cudaStream_t>(stream));
}
