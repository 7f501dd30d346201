// The two small GEMMs of a decode (layer, loop), with their element-wise tails fused:
//
//  writer   reg_out = bf16(reg_in + bf16(h . E^T))                          register.py:45-61
//           optionally committed in the epilogue: K half latent-RoPE'd in the torch bf16 order,
//           V half copied, row scattered to block_table[req, pos/page]*page + pos%page
//           (s6_layer.py:135-147 + unified_kv_cache_update, ouro_latent.py:127-129)
//  prepare  q_lat = latent_rope(bf16(q_pre . A_h))                           s6_layer.py:32-40
//           plus, in extra CTAs, the exact neox RoPE of q -> q_rope and of k, and the exact-cache
//           append of k_rope | v (model rotary_emb + unified_kv_cache_update, ouro_latent.py:113-123)
//
// Both are mma.m16n8k16 tiles fed by cp.async into XOR-swizzled shared memory (ldmatrix
// conflict-free).  A CTA computes 64 rows (tokens); each warp owns 16 of them.  Column tiles are
// chosen so one thread holds both members (i, i + w/2) of every neox RoPE pair it produces.
#include "common.cuh"
#include "decode_ops.cuh"
#include "gemm_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

// -------------------------------------------------------------------- writer (+ commit)
constexpr int kWKC = 128;     // k per stage
constexpr int kWStages = 4;
constexpr int kWRows = 64;    // tokens per CTA
constexpr int kWHBytes = kWRows * kWKC * 2;   // 16 KB
constexpr int kWEBytes = 16 * kWKC * 2;       // 4 KB

// Global column of element i (0..15) of column tile j.
__device__ __forceinline__ int writer_col(const WriterParams& p, int j, int i) {
  if (p.commit && j < p.w / 16) return (i < 8) ? 8 * j + i : p.w / 2 + 8 * j + (i - 8);
  if (p.commit) return p.w + 16 * (j - p.w / 16) + i;
  return 16 * j + i;
}

__global__ void __launch_bounds__(128) writer_kernel(const WriterParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int32_t qsl_s[kQslCap];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int j = blockIdx.x, t0 = blockIdx.y * kWRows;
  const int NK = p.K / kWKC;
  const int32_t* qsl = p.commit ? stage_qsl(p.qsl, p.R, qsl_s) : p.qsl;
  auto stage_h = [&](int s) { return smem + s * (kWHBytes + kWEBytes); };
  auto stage_e = [&](int s) { return smem + s * (kWHBytes + kWEBytes) + kWHBytes; };
  auto load = [&](int s, int kc) {
    const int k0 = kc * kWKC;
#pragma unroll
    for (int it = 0; it < 8; ++it) {  // h: 64 rows x 16 chunks
      const int idx = tid + it * 128, row = idx >> 4, ch = idx & 15;
      const int t = t0 + row;
      const __nv_bfloat16* src = p.h + static_cast<int64_t>(min(t, p.T - 1)) * p.h_st + k0 + ch * 8;
      cp_async16(stage_h(s) + swz(row, ch, 256), src, t < p.T ? 16 : 0);
    }
#pragma unroll
    for (int it = 0; it < 2; ++it) {  // E: 16 rows x 16 chunks
      const int idx = tid + it * 128, row = idx >> 4, ch = idx & 15;
      const int n = writer_col(p, j, row);
      cp_async16(stage_e(s) + swz(row, ch, 256), p.E + static_cast<int64_t>(n) * p.e_st + k0 + ch * 8);
    }
  };
#pragma unroll
  for (int s = 0; s < kWStages - 1; ++s) {
    if (s < NK) load(s, s);
    cp_async_commit();
  }
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int kc = 0; kc < NK; ++kc) {
    cp_async_wait<kWStages - 2>();
    __syncthreads();
    if (kc + kWStages - 1 < NK) load((kc + kWStages - 1) % kWStages, kc + kWStages - 1);
    cp_async_commit();
    const uint32_t hb = smem_u32(stage_h(kc % kWStages)), eb = smem_u32(stage_e(kc % kWStages));
#pragma unroll
    for (int ks = 0; ks < kWKC / 16; ++ks) {
      uint32_t a[4], b0, b1, b2, b3;
      const int arow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      ldsm_x4(hb + swz(arow, ks * 2 + (lane >> 4), 256), a[0], a[1], a[2], a[3]);
      const int brow = (lane & 7) + (lane >> 4) * 8;
      ldsm_x4(eb + swz(brow, ks * 2 + ((lane >> 3) & 1), 256), b0, b1, b2, b3);
      mma_bf16_16816(acc[0], a, b0, b1);
      mma_bf16_16816(acc[1], a, b2, b3);
    }
  }
  cp_async_wait<0>();

  // ---- epilogue: rows r0 = t0 + 16 warp + g and r0 + 8; columns 2c, 2c+1 of each n-tile
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int t = t0 + warp * 16 + g + half * 8;
    if (t >= p.T) continue;
    float u[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int col = writer_col(p, j, nt * 8 + 2 * c);
      u[nt][0] = bf16_round(acc[nt][2 * half]);
      u[nt][1] = bf16_round(acc[nt][2 * half + 1]);
      if (p.reg_in) {
        const __nv_bfloat162 r = *reinterpret_cast<const __nv_bfloat162*>(p.reg_in + static_cast<int64_t>(t) * p.ri_st + col);
        u[nt][0] = bf16_round(__bfloat162float(r.x) + u[nt][0]);
        u[nt][1] = bf16_round(__bfloat162float(r.y) + u[nt][1]);
      }
      if (p.reg_out)
        *reinterpret_cast<__nv_bfloat162*>(p.reg_out + static_cast<int64_t>(t) * p.ro_st + col) =
            __floats2bfloat162_rn(u[nt][0], u[nt][1]);
    }
    if (!p.commit) continue;
    const int64_t pos = p.positions[t];
    const int64_t slot = token_slot(qsl, p.R, t, pos, p.bt, p.bt_st, p.max_blocks, p.page, p.num_blocks);
    if (slot < 0) continue;
    __nv_bfloat16* dst = p.cache + (slot / p.page) * p.c_sb + (slot % p.page) * p.c_sr;
    if (j < p.w / 16) {
      const __nv_bfloat16* tab = p.table + clamp_pos(pos, p.max_pos) * p.tab_st;
      const int half_w = p.w / 2;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int a = 8 * j + 2 * c + e;  // pair (a, a + w/2)
        float y1, y2;
        rope_pair_torch(u[0][e], u[1][e], __bfloat162float(tab[a]), __bfloat162float(tab[half_w + a]), y1, y2);
        dst[a] = __float2bfloat16_rn(y1);
        dst[a + half_w] = __float2bfloat16_rn(y2);
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int col = writer_col(p, j, nt * 8 + 2 * c);
        *reinterpret_cast<__nv_bfloat162*>(dst + col) = __floats2bfloat162_rn(u[nt][0], u[nt][1]);
      }
    }
  }
}

int writer(const WriterParams& p, cudaStream_t s) {
  if (p.T == 0) return kStatusOk;
  if (writer_tc_eligible(p)) return writer_tc(p, s);  // prefill-size: tcgen05 tiles
  const int smem = kWStages * (kWHBytes + kWEBytes);
  static unsigned attr_mask = 0;
  ensure_smem_limit(writer_kernel, smem, attr_mask);
  dim3 grid(p.N / 16, (p.T + kWRows - 1) / kWRows);
  writer_kernel<<<grid, 128, smem, s>>>(p);
  return cuda_status(cudaGetLastError(), "writer_kernel launch");
}

// -------------------------------------------------------------------- prepare
// CTA x < W/64: latent query columns [32x, 32x+32) and their RoPE partners [W/2 + 32x, ...).
// CTAs x >= W/64 (when the exact part is enabled): exact RoPE + exact-cache append of head h,
// 16 tokens each, every load of a thread issued at once.  With exact_only the grid holds only those.
template <int W>
__global__ void __launch_bounds__(128) prepare_kernel(const PrepareParams p) {
  __shared__ __align__(128) uint8_t qs[64 * 256];   // q tile [64 tokens][128] bf16
  __shared__ __align__(128) uint8_t as[128 * 128];  // A tile [128 k][64 cols] bf16
  __shared__ __align__(16) __nv_bfloat16 cs_s[64][64];  // RoPE rows of the tile: [token][cos 32 | sin 32]
  __shared__ int64_t pos_s[64];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int x = blockIdx.x + (p.exact_only ? W / 64 : 0), h = blockIdx.y, t0 = blockIdx.z * 64;
  constexpr int HALF = W / 2;
  // a history split launched as this grid's programmatic dependent may start streaming pages now;
  // it reads q_lat only after this grid has completed.  Launched early itself (PrepareParams::pdl),
  // this grid touches memory only once the launch before it has completed.
  if (tid == 0) griddep_launch_dependents();
  griddep_wait();
  if (x >= W / 64) {
    const int32_t* qsl = stage_qsl(p.qsl, p.R, reinterpret_cast<int32_t*>(qs));  // q tile unused here
    // ---------------- exact part: 16 tokens of head h per CTA; thread = (token, 8 rotation pairs)
    const int tt = tid >> 3, i0 = (tid & 7) * 8;  // pairs i0..i0+7 with partners +64
    const int t = t0 + (x - W / 64) * 16 + tt;
    if (t >= p.T) return;
    const int64_t pos = p.positions[t];
    const float* cs = p.cos_sin + clamp_pos(pos, p.cs_max) * p.cs_st;
    const __nv_bfloat16* qp = p.q + static_cast<int64_t>(t) * p.q_st + static_cast<int64_t>(h) * p.q_sh;
    const __nv_bfloat16* kp = p.k + static_cast<int64_t>(t) * p.k_st + static_cast<int64_t>(h) * p.k_sh;
    const __nv_bfloat16* vp = p.v + static_cast<int64_t>(t) * p.v_st + static_cast<int64_t>(h) * p.v_sh;
    const float4 c0 = *reinterpret_cast<const float4*>(cs + i0), c1 = *reinterpret_cast<const float4*>(cs + i0 + 4);
    const float4 s0 = *reinterpret_cast<const float4*>(cs + 64 + i0), s1 = *reinterpret_cast<const float4*>(cs + 64 + i0 + 4);
    const uint4 qa = *reinterpret_cast<const uint4*>(qp + i0), qb = *reinterpret_cast<const uint4*>(qp + i0 + 64);
    const uint4 ka = *reinterpret_cast<const uint4*>(kp + i0), kb = *reinterpret_cast<const uint4*>(kp + i0 + 64);
    const uint4 va = *reinterpret_cast<const uint4*>(vp + i0), vb = *reinterpret_cast<const uint4*>(vp + i0 + 64);
    const float co[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float si[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const __nv_bfloat16* q1 = reinterpret_cast<const __nv_bfloat16*>(&qa);
    const __nv_bfloat16* q2 = reinterpret_cast<const __nv_bfloat16*>(&qb);
    const __nv_bfloat16* k1 = reinterpret_cast<const __nv_bfloat16*>(&ka);
    const __nv_bfloat16* k2 = reinterpret_cast<const __nv_bfloat16*>(&kb);
    uint4 qo1, qo2, ko1, ko2;
    __nv_bfloat16* qr1 = reinterpret_cast<__nv_bfloat16*>(&qo1);
    __nv_bfloat16* qr2 = reinterpret_cast<__nv_bfloat16*>(&qo2);
    __nv_bfloat16* kr1 = reinterpret_cast<__nv_bfloat16*>(&ko1);
    __nv_bfloat16* kr2 = reinterpret_cast<__nv_bfloat16*>(&ko2);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = __bfloat162float(q1[e]), b = __bfloat162float(q2[e]);
      qr1[e] = __float2bfloat16_rn(a * co[e] - b * si[e]);
      qr2[e] = __float2bfloat16_rn(b * co[e] + a * si[e]);
      const float ka_ = __bfloat162float(k1[e]), kb_ = __bfloat162float(k2[e]);
      kr1[e] = __float2bfloat16_rn(ka_ * co[e] - kb_ * si[e]);
      kr2[e] = __float2bfloat16_rn(kb_ * co[e] + ka_ * si[e]);
    }
    __nv_bfloat16* qr = p.q_rope + static_cast<int64_t>(t) * p.qr_st + static_cast<int64_t>(h) * p.qr_sh;
    *reinterpret_cast<uint4*>(qr + i0) = qo1;
    *reinterpret_cast<uint4*>(qr + i0 + 64) = qo2;
    const int64_t slot = token_slot(qsl, p.R, t, pos, p.bt, p.bt_st, p.max_blocks, p.page, p.num_blocks);
    if (p.slot_out && h == 0 && i0 == 0) p.slot_out[t] = slot;
    if (slot < 0) return;
    __nv_bfloat16* row_p = p.cache + (slot / p.page) * p.c_sb + static_cast<int64_t>(h) * p.c_sh +
                           (slot % p.page) * p.c_sr;
    *reinterpret_cast<uint4*>(row_p + i0) = ko1;
    *reinterpret_cast<uint4*>(row_p + i0 + 64) = ko2;
    *reinterpret_cast<uint4*>(row_p + 128 + i0) = va;
    *reinterpret_cast<uint4*>(row_p + 192 + i0) = vb;
    return;
  }
  // ---------------- latent query tile
  // one memory round for everything the tile reads: q, A and - once the positions are known - the RoPE
  // rows of the tile's 32 pair columns, all in flight together
  const int n0 = 32 * x;
  for (int idx = tid; idx < 64 * 16; idx += 128) {  // q: 64 rows x 16 chunks
    const int row = idx >> 4, ch = idx & 15, t = t0 + row;
    const __nv_bfloat16* src = p.q + static_cast<int64_t>(min(t, p.T - 1)) * p.q_st +
                               static_cast<int64_t>(h) * p.q_sh + ch * 8;
    cp_async16(qs + swz(row, ch, 256), src, t < p.T ? 16 : 0);
  }
  const __nv_bfloat16* Ah = p.A + static_cast<int64_t>(h) * p.a_sh;
  for (int idx = tid; idx < 128 * 8; idx += 128) {  // A: 128 k x (4 chunks low half, 4 chunks high half)
    const int k = idx >> 3, ch = idx & 7;
    const int col = ch < 4 ? n0 + ch * 8 : HALF + n0 + (ch - 4) * 8;
    cp_async16(as + swz(k, ch, 128), Ah + static_cast<int64_t>(k) * p.a_sk + col);
  }
  cp_async_commit();
  if (tid < 64) pos_s[tid] = t0 + tid < p.T ? clamp_pos(p.positions[t0 + tid], p.max_pos) : 0;
  __syncthreads();
  for (int idx = tid; idx < 64 * 8; idx += 128) {  // RoPE: 64 tokens x (4 cos chunks, 4 sin chunks)
    const int row = idx >> 3, ch = idx & 7;
    const __nv_bfloat16* tab = p.table + pos_s[row] * p.tab_st + (ch < 4 ? n0 + ch * 8 : HALF + n0 + (ch - 4) * 8);
    cp_async16(&cs_s[row][ch * 8], tab);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  float acc[8][4];
#pragma unroll
  for (int jn = 0; jn < 8; ++jn) acc[jn][0] = acc[jn][1] = acc[jn][2] = acc[jn][3] = 0.f;
  const uint32_t qb = smem_u32(qs), ab = smem_u32(as);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t a[4];
    const int arow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    ldsm_x4(qb + swz(arow, ks * 2 + (lane >> 4), 256), a[0], a[1], a[2], a[3]);
    const int krow = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(ab + swz(krow, 2 * jp + (lane >> 4), 128), b0, b1, b2, b3);
      mma_bf16_16816(acc[2 * jp], a, b0, b1);
      mma_bf16_16816(acc[2 * jp + 1], a, b2, b3);
    }
  }
  // tile column of n-tile jn: jn < 4 -> n0 + 8 jn (+2c), jn >= 4 -> HALF + n0 + 8 (jn - 4)
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = warp * 16 + g + half * 8, t = t0 + row;
    if (t >= p.T) continue;
    __nv_bfloat16* dst = p.q_lat + static_cast<int64_t>(t) * p.ql_st + static_cast<int64_t>(h) * p.ql_sh;
#pragma unroll
    for (int jn = 0; jn < 4; ++jn) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int a = n0 + 8 * jn + 2 * c + e, la = 8 * jn + 2 * c + e;  // la: column within the tile's 32
        float y1, y2;
        rope_pair_torch(bf16_round(acc[jn][2 * half + e]), bf16_round(acc[jn + 4][2 * half + e]),
                        __bfloat162float(cs_s[row][la]), __bfloat162float(cs_s[row][32 + la]), y1, y2);
        dst[a] = __float2bfloat16_rn(y1);
        dst[a + HALF] = __float2bfloat16_rn(y2);
      }
    }
  }
}

int prepare(const PrepareParams& p, cudaStream_t s) {
  if (p.T == 0) return kStatusOk;
  const int extra = p.k ? 4 : 0;  // exact-part CTAs per (head, 64-token block): 16 tokens each
  if (p.exact_only && !p.k) {
    set_error("prepare: the exact part alone needs k");
    return kStatusInvalid;
  }
  dim3 grid(p.exact_only ? extra : p.W / 64 + extra, p.H, (p.T + 63) / 64);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.pdl ? 1 : 0;
  cudaError_t e;
  switch (p.W) {
    case 256: e = cudaLaunchKernelEx(&cfg, prepare_kernel<256>, p); break;
    case 512: e = cudaLaunchKernelEx(&cfg, prepare_kernel<512>, p); break;
    case 1024: e = cudaLaunchKernelEx(&cfg, prepare_kernel<1024>, p); break;
    default: set_error("latent query width %d unsupported (256, 512, 1024)", p.W); return kStatusInvalid;
  }
  return cuda_status(e, "prepare_kernel launch");
}

}  // namespace hla
