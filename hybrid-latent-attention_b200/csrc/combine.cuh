// Argument block of the fused decode combine (combine.cu).
#pragma once
#include "decode_ops.cuh"

namespace hla {

struct CombineParams {
  // history input: split partials of the history kernel (ws_o / ws_lse / meta as planned for the
  // same call) or, when z_in is set, num_parts reduced partials (fp32 z and its lse) - one per GPU
  // of a sequence-split history - that are LSE-merged here
  const float* ws_o;
  const float* ws_lse;
  const int2* meta;
  int stream_mode;
  const float* z_in;    // part q: z [T, H, W] at z_in + q * part_stride
  const float* lse_in;  // part q: lse [H, T] at lse_in + q * part_stride
  // or the parts as exchange words (8 bytes per value, part_stride counting words) stored by other
  // GPUs' history_reduce_exchange: polled until tagged *epoch + 1; the last CTA through advances
  // *epoch and re-zeroes part_seen (a count of the CTAs)
  const uint64_t* zw_in;
  const uint64_t* lw_in;
  int num_parts;
  int64_t part_stride;
  int* epoch;
  int* part_seen;
  int* err;  // optional device error word (a peer that never delivers)
  uint64_t wait_ns;  // bound of the exchange-word polls and of the B-load wait (device ns)
  const uint8_t* empty;  // optional [T]: rows whose latent history is empty
  int T, H;
  const __nv_bfloat16* B;  // [H, W, 128] up-projection
  int64_t b_sh, b_sk;
  WindowArgs win;
  // external exact part (prefill / mixed steps): the chunk attention already merged with the window
  // history, used in place of the decode window when chunk_o is set
  const __nv_bfloat16* chunk_o;
  int64_t co_st, co_sh;
  const float* chunk_lse;
  __nv_bfloat16* out;  // [T, H, 128]
  int64_t o_st, o_sh;
  float* lse_out;  // optional [H, T] merged lse
};

// pdl: launch as a programmatic dependent of the immediately preceding launch on `s`, which must
// be the history split kernel that produced the partials (the window part then overlaps its tail).
int decode_combine(const CombineParams& p, int W, bool pdl, cudaStream_t s);

}  // namespace hla
