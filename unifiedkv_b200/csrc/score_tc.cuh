// Parameters of the tcgen05 scoring passes of the block-aligned SnapKV
// compression (compress_tc.cu), shared with their caller in compress.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace bpkv {

struct ScoreTcParams {
  const void* k;
  const void* q;
  int Hkv, n_rep, W, Wp, Lm, Tm, sink;
  int n_chunks;         // in: partial-stat slots per window row in the workspace; out: ranges per KV group
  int tiles_per_chunk;  // out (pass 1): 128-token K tiles per range
  int hm_slots;         // out (pass 2): headmax rows per KV group (one per head slot; max taken later)
  int64_t k_sh, k_st, q_sh, q_st;
  float scale_log2;
  float2* ml_part;   // [Hq*Wp][n_chunks] (m in log2 units, l)
  const float2* ml;  // [Hq*Wp]
  float* headmax;    // [Hkv * hm_slots][Tm]
};

// Pass 1 (row statistics) or pass 2 (per-token head max) on tcgen05 when the shape
// allows (head_dim 128, <= 256 window rows per KV group, bf16 / fp16, 16-byte K
// strides); BPKV_ERR_UNSUPPORTED otherwise.  Pass 1 sets n_chunks and tiles_per_chunk
// for the stats reduction and for pass 2, which must get the same struct.
int score_tc_pass(ScoreTcParams& p, int head_dim, int dtype, int pass, cudaStream_t st);

}  // namespace bpkv
