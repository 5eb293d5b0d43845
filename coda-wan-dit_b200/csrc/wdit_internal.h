// Internal structures shared by the CUDA translation units (not part of the C ABI).
#pragma once
#include "../../include/wdit.h"

namespace wdit {

struct GemmShape {
  int M, N, K;
  int m_blocks, n_blocks, k_blocks, tiles;
};

// adaLN LayerNorm absorbed into a GEMM:  rstd * (acc - mu * csum[n]).
struct LnFold {
  const float* csum;   // [N] column sums of the folded weight; nullptr = no LayerNorm
  const float* stats;  // [M, stats_tiles, 2] per-tile (mean, M2) partials of the input rows
  int stats_tiles;
  int stats_width;     // columns per partial
  int row_len;         // normalized row length (= K)
  float eps;
};

struct EpiParams {
  const float* vec;  // per-column bias / shift term [N], nullable
  LnFold ln;
  int act;  // kEpiAct: 0 = identity, 1 = tanh-GELU
  // residual epilogue
  const float* gate_a;  // [N], nullable (no gate)
  const float* gate_b;  // [batches, gate_b_stride], nullable; gate = gate_a + gate_b[batch]
  int gate_b_stride;
  int rows_per_batch;  // rows of one batch entry along M (per-batch vectors, RoPE token index)
  float* stats_out;    // [M, ceil(N/256), 2], nullable
  // norm epilogue
  int norm_groups;  // leading column groups of width norm_width that get the full-width RMSNorm
  int norm_width;
  const float* norm_w[2];
  float norm_eps;
  int rope_groups;  // leading groups that also get 3D RoPE
  const float* rope_cos;
  const float* rope_sin;
  int rope_ld;  // pair-major tables: entry (pair, token) at pair * rope_ld + token
  int token_offset;
  float* part;             // scratch [M, norm_groups * norm_width/256]
  unsigned int* counters;  // scratch [m_blocks * norm_groups], zero between launches
  void* out;  // norm epilogue: direct bf16 stores
  int ldo;
  void* x_out;  // residual epilogue: bf16 copy of the result (direct stores)
  int ldx;
  int has_out_map;
  int has_x_map;
};

}  // namespace wdit
