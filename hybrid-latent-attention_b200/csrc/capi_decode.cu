// Exported C entry points of the decode ops around the history reader (include/hla_s6.h).
#include "../../include/hla_s6.h"
#include "combine.cuh"
#include "decode_ops.cuh"
#include "gemm_ops.cuh"
#include "hla_s6_internal.h"

namespace hla {

static bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

static int check_window(const WindowArgs& w, int head_dim) {
  if (head_dim != 128) {
    set_error("exact window kernel is built for head_dim 128 (got %d)", head_dim);
    return kStatusInvalid;
  }
  if (w.window < 0 || w.window > 127) {
    set_error("window %d unsupported (0..127)", w.window);
    return kStatusInvalid;
  }
  if (w.page < 1 || !aligned(w.cache, 16) || (w.c_sb % 8) || (w.c_sh % 8) || (w.c_sr % 8)) {
    set_error("exact cache needs a 16-byte aligned base and strides that are multiples of 8 elements");
    return kStatusInvalid;
  }
  if (!aligned(w.q, 8) || (w.q_st % 4) || (w.q_sh % 4)) {
    set_error("q needs 8-byte aligned rows (strides multiples of 4) and a unit last-dim stride");
    return kStatusInvalid;
  }
  return kStatusOk;
}

static WindowArgs make_window(const void* q, int64_t q_st, int64_t q_sh, const void* cache, int64_t num_blocks,
                              int64_t c_sb, int64_t c_sh, int64_t c_sr, int32_t page, const int32_t* bt,
                              int64_t bt_st, int32_t max_blocks, const int32_t* qsl, int32_t R,
                              const int32_t* seq_lens, int32_t window, float scale) {
  WindowArgs w;
  w.q = static_cast<const __nv_bfloat16*>(q);
  w.q_st = q_st;
  w.q_sh = q_sh;
  w.cache = static_cast<const __nv_bfloat16*>(cache);
  w.c_sb = c_sb;
  w.c_sh = c_sh;
  w.c_sr = c_sr;
  w.num_blocks = num_blocks;
  w.page = page;
  w.bt = bt;
  w.bt_st = bt_st;
  w.max_blocks = max_blocks;
  w.qsl = qsl;
  w.R = R;
  w.seq_lens = seq_lens;
  w.window = window;
  w.scale = scale;
  w.ctx_tok = nullptr;
  return w;
}

}  // namespace hla

using namespace hla;

extern "C" {

int hla_s6_window_attention(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                            int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                            int64_t cache_stride_row, int32_t page, const int32_t* block_table,
                            int64_t block_table_stride, int32_t max_blocks, const int32_t* query_start_loc,
                            int32_t num_reqs, const int32_t* seq_lens, int32_t window, float scale,
                            int32_t num_tokens, int32_t num_heads, int32_t head_dim, void* out, int64_t out_stride_t,
                            int64_t out_stride_h, float* lse, void* stream) {
  WindowArgs w = make_window(q, q_stride_t, q_stride_h, cache, num_blocks, cache_stride_block, cache_stride_head,
                             cache_stride_row, page, block_table, block_table_stride, max_blocks, query_start_loc,
                             num_reqs, seq_lens, window, scale);
  int rc = check_window(w, head_dim);
  if (rc) return rc;
  if (num_reqs < 1) {
    set_error("window attention needs at least one request");
    return kStatusInvalid;
  }
  return window_attention(w, num_tokens, num_heads, out, out_stride_t, out_stride_h, lse,
                          static_cast<cudaStream_t>(stream));
}

int hla_s6_window_history(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* cache,
                          int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                          int64_t cache_stride_row, int32_t page, const int32_t* token_block_table,
                          int64_t block_table_stride, int32_t max_blocks, const int32_t* ctx, int32_t window,
                          float scale, int32_t num_tokens, int32_t num_heads, int32_t head_dim, void* out,
                          int64_t out_stride_t, int64_t out_stride_h, float* lse, void* stream) {
  WindowArgs w = make_window(q, q_stride_t, q_stride_h, cache, num_blocks, cache_stride_block, cache_stride_head,
                             cache_stride_row, page, token_block_table, block_table_stride, max_blocks, nullptr, 0,
                             nullptr, window, scale);
  w.ctx_tok = ctx;
  int rc = check_window(w, head_dim);
  if (rc) return rc;
  return window_attention(w, num_tokens, num_heads, out, out_stride_t, out_stride_h, lse,
                          static_cast<cudaStream_t>(stream));
}

int hla_s6_merge_states(const void* o_hist, int64_t hist_stride_t, int64_t hist_stride_h, const float* lse_hist,
                        const void* o_chunk, int64_t chunk_stride_t, int64_t chunk_stride_h, const float* lse_chunk,
                        const uint8_t* invalid, void* out, int64_t out_stride_t, int64_t out_stride_h,
                        int32_t num_tokens, int32_t num_heads, int32_t dim, void* stream) {
  return merge(o_hist, hist_stride_t, hist_stride_h, lse_hist, o_chunk, chunk_stride_t, chunk_stride_h, lse_chunk,
               invalid, out, out_stride_t, out_stride_h, nullptr, num_tokens, num_heads, dim, 0,
               static_cast<cudaStream_t>(stream));
}

int hla_s6_merge_lse(const void* o1, int64_t o1_stride_t, int64_t o1_stride_h, const float* lse1, const void* o2,
                     int64_t o2_stride_t, int64_t o2_stride_h, const float* lse2, void* out, int64_t out_stride_t,
                     int64_t out_stride_h, float* lse_out, int32_t num_tokens, int32_t num_heads, int32_t dim,
                     void* stream) {
  return merge(o1, o1_stride_t, o1_stride_h, lse1, o2, o2_stride_t, o2_stride_h, lse2, nullptr, out, out_stride_t,
               out_stride_h, lse_out, num_tokens, num_heads, dim, 1, static_cast<cudaStream_t>(stream));
}

int hla_s6_latent_rope(void* x, int64_t x_stride_t, int64_t x_stride_h, int32_t num_tokens, int32_t num_heads,
                       int32_t width, const int64_t* positions, const void* table, int64_t table_stride,
                       int64_t max_position, void* stream) {
  if (width < 2 || (width % 2) || max_position < 1 || table_stride < width) {
    set_error("latent rope needs an even width and a [max_position, width] table");
    return kStatusInvalid;
  }
  return latent_rope(x, x_stride_t, x_stride_h, num_tokens, num_heads, width, positions, table, table_stride,
                     max_position, static_cast<cudaStream_t>(stream));
}

int hla_s6_latent_query(const void* q_pre, int64_t q_stride_t, int64_t q_stride_h, const void* A, int64_t a_stride_h,
                        int64_t a_stride_k, const int64_t* positions, const void* table, int64_t table_stride,
                        int64_t max_position, void* out, int64_t out_stride_t, int64_t out_stride_h,
                        int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t width, void* stream) {
  return hla_s6_decode_prepare(q_pre, q_stride_t, q_stride_h, A, a_stride_h, a_stride_k, positions, table,
                               table_stride, max_position, out, out_stride_t, out_stride_h, num_tokens, num_heads,
                               head_dim, width, nullptr, 0, 0, nullptr, 0, 0, nullptr, 0, 0, nullptr, 0, 0, nullptr, 0,
                               0, 0, 0, 0, nullptr, 0, 0, nullptr, 0, nullptr, 0, stream);
}

int hla_s6_decode_prepare(const void* q_pre, int64_t q_stride_t, int64_t q_stride_h, const void* A,
                          int64_t a_stride_h, int64_t a_stride_k, const int64_t* positions, const void* table,
                          int64_t table_stride, int64_t max_position, void* q_lat, int64_t q_lat_stride_t,
                          int64_t q_lat_stride_h, int32_t num_tokens, int32_t num_heads, int32_t head_dim,
                          int32_t width, void* q_rope, int64_t q_rope_stride_t, int64_t q_rope_stride_h,
                          const void* k, int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                          int64_t v_stride_h, const float* cos_sin, int64_t cos_sin_stride, int64_t cos_sin_rows,
                          void* cache, int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                          int64_t cache_stride_row, int32_t page, const int32_t* block_table,
                          int64_t block_table_stride, int32_t max_blocks, const int32_t* query_start_loc,
                          int32_t num_reqs, int64_t* slot_out, int32_t flags, void* stream) {
  if (head_dim != 128 || (width != 256 && width != 512 && width != 1024)) {
    set_error("latent query needs head_dim 128 and width 256, 512 or 1024 (got %d, %d)", head_dim, width);
    return kStatusInvalid;
  }
  if (max_position < 1 || table_stride < width || !aligned(table, 16) || (table_stride % 8) || !aligned(q_pre, 16) ||
      (q_stride_t % 8) || (q_stride_h % 8) || !aligned(A, 16) || (a_stride_h % 8) || (a_stride_k % 8)) {
    set_error("latent query needs a [max_position, width] table and 16-byte aligned table / q / A rows");
    return kStatusInvalid;
  }
  if (k && (page < 1 || num_reqs < 1 || cos_sin_rows < 1 || cos_sin_stride < 128 || (cos_sin_stride % 4) || !q_rope ||
            !aligned(cos_sin, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(q_rope, 16) || !aligned(cache, 16) ||
            (k_stride_t % 8) || (k_stride_h % 8) || (v_stride_t % 8) || (v_stride_h % 8) || (q_rope_stride_t % 8) ||
            (q_rope_stride_h % 8) || (cache_stride_block % 8) || (cache_stride_head % 8) || (cache_stride_row % 8))) {
    set_error("exact part needs page >= 1, >= 1 request, a 16-byte aligned [max_position, 128] cos|sin table, a q_rope "
              "buffer and 16-byte aligned rows of k, v, q_rope and the exact cache");
    return kStatusInvalid;
  }
  PrepareParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q_pre);
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.A = static_cast<const __nv_bfloat16*>(A);
  p.a_sh = a_stride_h;
  p.a_sk = a_stride_k;
  p.positions = positions;
  p.table = static_cast<const __nv_bfloat16*>(table);
  p.tab_st = table_stride;
  p.max_pos = max_position;
  p.q_lat = static_cast<__nv_bfloat16*>(q_lat);
  p.ql_st = q_lat_stride_t;
  p.ql_sh = q_lat_stride_h;
  p.T = num_tokens;
  p.H = num_heads;
  p.W = width;
  p.q_rope = static_cast<__nv_bfloat16*>(q_rope);
  p.qr_st = q_rope_stride_t;
  p.qr_sh = q_rope_stride_h;
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.k_st = k_stride_t;
  p.k_sh = k_stride_h;
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.v_st = v_stride_t;
  p.v_sh = v_stride_h;
  p.cos_sin = cos_sin;
  p.cs_st = cos_sin_stride;
  p.cs_max = cos_sin_rows;
  p.cache = static_cast<__nv_bfloat16*>(cache);
  p.c_sb = cache_stride_block;
  p.c_sh = cache_stride_head;
  p.c_sr = cache_stride_row;
  p.num_blocks = num_blocks;
  p.page = page;
  p.bt = block_table;
  p.bt_st = block_table_stride;
  p.max_blocks = max_blocks;
  p.qsl = query_start_loc;
  p.R = num_reqs;
  p.slot_out = slot_out;
  p.pdl = (flags & HLA_S6_PREPARE_EARLY_LAUNCH) != 0;
  p.exact_only = (flags & HLA_S6_PREPARE_EXACT_ONLY) != 0;
  return prepare(p, static_cast<cudaStream_t>(stream));
}

int hla_s6_exact_append(void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                        int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h, void* k_out,
                        int64_t k_out_stride_t, int64_t k_out_stride_h, const int64_t* positions,
                        const float* cos_sin, int64_t cos_sin_stride, int64_t max_position, void* cache,
                        int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_head,
                        int64_t cache_stride_row, int32_t page, const int32_t* block_table, int64_t block_table_stride,
                        int32_t max_blocks, const int32_t* query_start_loc, int32_t num_reqs, int32_t num_tokens,
                        int32_t num_heads, int32_t head_dim, int64_t* slot_out, void* stream) {
  if (head_dim != 128 || page < 1 || num_reqs < 1 || max_position < 1 || cos_sin_stride < 128) {
    set_error("exact append needs head_dim 128, page >= 1, >= 1 request and a [max_position, 128] cos|sin table");
    return kStatusInvalid;
  }
  ExactArgs a;
  a.q = static_cast<__nv_bfloat16*>(q);
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.k_st = k_stride_t;
  a.k_sh = k_stride_h;
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.v_st = v_stride_t;
  a.v_sh = v_stride_h;
  a.k_out = static_cast<__nv_bfloat16*>(k_out);
  a.ko_st = k_out_stride_t;
  a.ko_sh = k_out_stride_h;
  a.positions = positions;
  a.cos_sin = cos_sin;
  a.cs_st = cos_sin_stride;
  a.max_pos = max_position;
  a.cache = static_cast<__nv_bfloat16*>(cache);
  a.c_sb = cache_stride_block;
  a.c_sh = cache_stride_head;
  a.c_sr = cache_stride_row;
  a.num_blocks = num_blocks;
  a.page = page;
  a.bt = block_table;
  a.bt_st = block_table_stride;
  a.max_blocks = max_blocks;
  a.qsl = query_start_loc;
  a.R = num_reqs;
  a.H = num_heads;
  a.slot_out = slot_out;
  return exact_append(a, num_tokens, static_cast<cudaStream_t>(stream));
}

static int writer_checks(const void* h, int64_t h_st, const void* E, int64_t e_st, const void* reg_in,
                         int64_t ri_st, const void* reg_out, int64_t ro_st, int32_t N, int32_t K) {
  if (K % 128 || N % 16 || !aligned(h, 16) || (h_st % 8) || !aligned(E, 16) || (e_st % 8) ||
      (reg_in && ((ri_st % 2) || !aligned(reg_in, 4))) || (reg_out && ((ro_st % 2) || !aligned(reg_out, 4)))) {
    set_error("writer needs in_features % 128 == 0, out_features % 16 == 0, 16-byte aligned h / weight rows "
              "and even register strides");
    return kStatusInvalid;
  }
  return kStatusOk;
}

int hla_s6_writer_project(const void* h, int64_t h_stride_t, const void* weight, int64_t weight_stride_n,
                          const void* reg_in, int64_t reg_in_stride_t, void* reg_out, int64_t reg_out_stride_t,
                          int32_t num_tokens, int32_t out_features, int32_t in_features, void* stream) {
  int rc = writer_checks(h, h_stride_t, weight, weight_stride_n, reg_in, reg_in_stride_t, reg_out,
                         reg_out_stride_t, out_features, in_features);
  if (rc) return rc;
  if (!reg_out) {
    set_error("writer projection needs an output register");
    return kStatusInvalid;
  }
  WriterParams p{};
  p.h = static_cast<const __nv_bfloat16*>(h);
  p.h_st = h_stride_t;
  p.E = static_cast<const __nv_bfloat16*>(weight);
  p.e_st = weight_stride_n;
  p.reg_in = static_cast<const __nv_bfloat16*>(reg_in);
  p.ri_st = reg_in_stride_t;
  p.reg_out = static_cast<__nv_bfloat16*>(reg_out);
  p.ro_st = reg_out_stride_t;
  p.T = num_tokens;
  p.N = out_features;
  p.K = in_features;
  return writer(p, static_cast<cudaStream_t>(stream));
}

int hla_s6_writer_commit(const void* h, int64_t h_stride_t, const void* weight, int64_t weight_stride_n,
                         const void* reg_in, int64_t reg_in_stride_t, void* reg_out, int64_t reg_out_stride_t,
                         int32_t num_tokens, int32_t out_features, int32_t in_features, const int64_t* positions,
                         const void* table, int64_t table_stride, int64_t max_position, void* cache,
                         int64_t num_blocks, int64_t cache_stride_block, int64_t cache_stride_row, int32_t page,
                         const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                         const int32_t* query_start_loc, int32_t num_reqs, void* stream) {
  int rc = writer_checks(h, h_stride_t, weight, weight_stride_n, reg_in, reg_in_stride_t, reg_out,
                         reg_out_stride_t, out_features, in_features);
  if (rc) return rc;
  const int w = out_features / 2;
  if (w % 16 || page < 1 || num_reqs < 1 || max_position < 1 || table_stride < w) {
    set_error("writer commit needs width % 16 == 0, page >= 1, >= 1 request and a [max_position, width] table");
    return kStatusInvalid;
  }
  WriterParams p{};
  p.h = static_cast<const __nv_bfloat16*>(h);
  p.h_st = h_stride_t;
  p.E = static_cast<const __nv_bfloat16*>(weight);
  p.e_st = weight_stride_n;
  p.reg_in = static_cast<const __nv_bfloat16*>(reg_in);
  p.ri_st = reg_in_stride_t;
  p.reg_out = static_cast<__nv_bfloat16*>(reg_out);
  p.ro_st = reg_out_stride_t;
  p.T = num_tokens;
  p.N = out_features;
  p.K = in_features;
  p.commit = 1;
  p.w = w;
  p.positions = positions;
  p.table = static_cast<const __nv_bfloat16*>(table);
  p.tab_st = table_stride;
  p.max_pos = max_position;
  p.cache = static_cast<__nv_bfloat16*>(cache);
  p.c_sb = cache_stride_block;
  p.c_sr = cache_stride_row;
  p.num_blocks = num_blocks;
  p.page = page;
  p.bt = block_table;
  p.bt_st = block_table_stride;
  p.max_blocks = max_blocks;
  p.qsl = query_start_loc;
  p.R = num_reqs;
  return writer(p, static_cast<cudaStream_t>(stream));
}

int hla_s6_commit_rows(const void* row, int64_t row_stride_t, int32_t width, const int64_t* positions,
                       const void* table, int64_t table_stride, int64_t max_position, void* cache, int64_t num_blocks,
                       int64_t cache_stride_block, int64_t cache_stride_row, int32_t page, const int32_t* block_table,
                       int64_t block_table_stride, int32_t max_blocks, const int32_t* query_start_loc,
                       int32_t num_reqs, int32_t num_tokens, int64_t* slot_out, void* stream) {
  if (width < 2 || (width % 2) || page < 1 || num_reqs < 1 || max_position < 1 || table_stride < width) {
    set_error("commit rows needs an even width, page >= 1, >= 1 request and a [max_position, width] table");
    return kStatusInvalid;
  }
  CommitArgs a;
  a.row = static_cast<const __nv_bfloat16*>(row);
  a.row_st = row_stride_t;
  a.w = width;
  a.positions = positions;
  a.table = static_cast<const __nv_bfloat16*>(table);
  a.tab_st = table_stride;
  a.max_pos = max_position;
  a.cache = static_cast<__nv_bfloat16*>(cache);
  a.c_sb = cache_stride_block;
  a.c_sr = cache_stride_row;
  a.num_blocks = num_blocks;
  a.page = page;
  a.bt = block_table;
  a.bt_st = block_table_stride;
  a.max_blocks = max_blocks;
  a.qsl = query_start_loc;
  a.R = num_reqs;
  a.slot_out = slot_out;
  return commit_rows(a, num_tokens, static_cast<cudaStream_t>(stream));
}

int hla_s6_decode_combine(int32_t num_tokens, int32_t num_heads, int32_t width, int32_t latent_page,
                          int32_t num_kv_splits, float* workspace, int64_t workspace_floats, const void* z_in,
                          const void* lse_in, int32_t num_parts, int64_t part_stride, int32_t* epoch,
                          int32_t* part_seen, const uint8_t* empty,
                          const void* B, int64_t b_stride_h,
                          int64_t b_stride_k, const void* q_rope, int64_t q_stride_t, int64_t q_stride_h,
                          const void* exact_cache, int64_t exact_num_blocks, int64_t exact_stride_block,
                          int64_t exact_stride_head, int64_t exact_stride_row, int32_t exact_page,
                          const int32_t* block_table, int64_t block_table_stride, int32_t max_blocks,
                          const int32_t* query_start_loc, int32_t num_reqs, const int32_t* seq_lens, int32_t window,
                          float scale, const void* chunk_o, int64_t chunk_stride_t, int64_t chunk_stride_h,
                          const float* chunk_lse, void* out, int64_t out_stride_t, int64_t out_stride_h,
                          float* lse_out, int32_t flags, int* error_flag, void* stream) {
  CombineParams p;
  p.win = make_window(q_rope, q_stride_t, q_stride_h, exact_cache, exact_num_blocks, exact_stride_block,
                      exact_stride_head, exact_stride_row, exact_page, block_table, block_table_stride, max_blocks,
                      query_start_loc, num_reqs, seq_lens, window, scale);
  int rc = kStatusOk;
  if (chunk_o) {
    if (!chunk_lse || !aligned(chunk_o, 8) || (chunk_stride_t % 4) || (chunk_stride_h % 4)) {
      set_error("decode combine: an external chunk part needs 8-byte aligned rows and its lse");
      return kStatusInvalid;
    }
  } else if ((rc = check_window(p.win, 128))) {
    return rc;
  }
  p.chunk_o = static_cast<const __nv_bfloat16*>(chunk_o);
  p.co_st = chunk_stride_t;
  p.co_sh = chunk_stride_h;
  p.chunk_lse = chunk_lse;
  if (num_heads < 1 || num_heads > 16 || num_reqs < 1) {
    set_error("decode combine needs 1..16 heads and >= 1 request");
    return kStatusInvalid;
  }
  if ((out_stride_t % 2) || (out_stride_h % 2)) {
    set_error("decode combine output needs even strides");
    return kStatusInvalid;
  }
  HistoryPlan plan{};
  if (!z_in) {
    HistoryArgs a{};
    a.T = num_tokens;
    a.H = num_heads;
    a.W = width;
    a.page = latent_page;
    a.num_kv_splits = num_kv_splits;
    a.ws = workspace;
    a.ws_floats = workspace_floats;
    a.waves = 1;
    if ((rc = history_plan(a, &plan))) return rc;
  } else if (!lse_in || !aligned(z_in, 16) || num_parts < 1 ||
             (num_parts > 1 && (part_stride % (epoch ? 2 : 4)))) {
    set_error("a reduced history input needs >= 1 part of 16-byte aligned z [T, H, W] with its lse [H, T] "
              "(part stride a multiple of 4 floats, or of 2 exchange words)");
    return kStatusInvalid;
  }
  if (epoch && (!z_in || !part_seen || num_parts > 32 || !aligned(lse_in, 8))) {
    set_error("decode combine: exchange words need reduced parts (z_in, 8-byte aligned lse_in, <= 32 parts), "
              "the slot's epoch counter and a CTA counter");
    return kStatusInvalid;
  }
  p.ws_o = plan.ws_o;
  p.ws_lse = plan.ws_lse;
  p.meta = plan.meta;
  p.stream_mode = plan.stream_mode;
  p.z_in = epoch ? nullptr : static_cast<const float*>(z_in);
  p.lse_in = epoch ? nullptr : static_cast<const float*>(lse_in);
  p.zw_in = epoch ? static_cast<const uint64_t*>(z_in) : nullptr;
  p.lw_in = epoch ? static_cast<const uint64_t*>(lse_in) : nullptr;
  p.num_parts = z_in ? num_parts : 0;
  p.part_stride = part_stride;
  p.epoch = epoch;
  p.part_seen = part_seen;
  p.err = error_flag;
  p.wait_ns = wait_limit_ns();
  p.empty = empty;
  p.T = num_tokens;
  p.H = num_heads;
  p.B = static_cast<const __nv_bfloat16*>(B);
  p.b_sh = b_stride_h;
  p.b_sk = b_stride_k;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_st = out_stride_t;
  p.o_sh = out_stride_h;
  p.lse_out = lse_out;
  const bool pdl = (flags & HLA_S6_COMBINE_AFTER_PARTIALS) != 0;
  return decode_combine(p, width, pdl, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
