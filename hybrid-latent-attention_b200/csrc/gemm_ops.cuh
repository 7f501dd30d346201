// Argument blocks of the writer and prepare kernels (gemm_ops.cu).
#pragma once
#include "common.cuh"

namespace hla {

struct WriterParams {
  const __nv_bfloat16* h;  // [T, K] attention input of this loop
  int64_t h_st;
  const __nv_bfloat16* E;  // [N, K] writer weight (nn.Linear layout)
  int64_t e_st;
  const __nv_bfloat16* reg_in;  // [T, N] running register (NULL at its first loop)
  int64_t ri_st;
  __nv_bfloat16* reg_out;  // [T, N] (NULL: commit only)
  int64_t ro_st;
  int T, N, K;
  // commit (N == 2 w): K half latent-RoPE'd, row scattered into the latent cache
  int commit, w;
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
  int* err;  // optional device error word (bounded waits of the tcgen05 path)
  uint64_t wait_ns;  // bound of every mbarrier wait of the tcgen05 path (device ns)
};

struct PrepareParams {
  const __nv_bfloat16* q;  // pre-RoPE q [T, H, 128]
  int64_t q_st, q_sh;
  const __nv_bfloat16* A;  // [H, 128, W]
  int64_t a_sh, a_sk;
  const int64_t* positions;
  const __nv_bfloat16* table;  // latent [max_pos, W] = [cos | sin]
  int64_t tab_st, max_pos;
  __nv_bfloat16* q_lat;  // [T, H, W]
  int64_t ql_st, ql_sh;
  int T, H, W;
  // exact part (enabled when k != NULL)
  __nv_bfloat16* q_rope;  // [T, H, 128] exact-RoPE'd q
  int64_t qr_st, qr_sh;
  const __nv_bfloat16* k;
  int64_t k_st, k_sh;
  const __nv_bfloat16* v;
  int64_t v_st, v_sh;
  const float* cos_sin;  // [max_pos, 128] = [cos 64 | sin 64] fp32
  int64_t cs_st, cs_max;
  __nv_bfloat16* cache;  // exact cache, logical [nb, H, page, 256]
  int64_t c_sb, c_sh, c_sr, num_blocks;
  int page;
  const int32_t* bt;
  int64_t bt_st;
  int max_blocks;
  const int32_t* qsl;
  int R;
  int64_t* slot_out;
  bool pdl;  // launch as a programmatic dependent of the preceding launch (the kernel waits for it)
  bool exact_only;  // run only the exact part's CTAs (k != NULL): no latent query, q_lat untouched
};

int writer(const WriterParams& p, cudaStream_t s);
bool writer_tc_eligible(const WriterParams& p);  // writer_tc.cu
int writer_tc(const WriterParams& p, cudaStream_t s);
int prepare(const PrepareParams& p, cudaStream_t s);

}  // namespace hla
