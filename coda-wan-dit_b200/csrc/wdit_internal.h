// Internal structures shared by the CUDA translation units (not part of the C ABI).
#pragma once
#include "../../include/wdit.h"

namespace wdit {

struct GemmShape {
  int M, N, K;
  int m_blocks, n_blocks, k_blocks, tiles;
  // Unit schedule of the norm GEMM (kEpiNorm; zero otherwise): the leading norm_groups column
  // groups of `unit_tiles` N tiles each are processed one (row block, group) unit at a time by
  // one CTA (pair); the remaining `plain_nblocks` N tiles of every row block are plain tiles.
  int norm_groups, unit_tiles, plain_nblocks, units;
  int raster_rows;  // row blocks per rasterization group (1 = row-major tile order)
};

// Full-width RMSNorm (+ RoPE) applied by the norm GEMM's epilogue (kEpiNorm).
struct NormParams {
  void* out;            // bf16 output (the GEMM's), rows of ldo elements
  int ldo;
  int width;            // columns per normalized group (multiple of 256)
  float inv_width;
  float eps;
  const float* w0;      // RMSNorm weight of group 0 [width]
  const float* w1;      // ... of group 1 (norm_groups == 2)
  int rope_groups;      // leading groups that also get the RoPE rotation
  const float* cos;     // token-major [tokens, rope_ld] fp32 tables
  const float* sin;
  int rope_ld;
  int token_offset;     // token of row m: m % rows_per_batch + token_offset
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

// Token-sharded runs: the norm GEMM sends its results straight into the ranks' exchange
// regions (the Ulysses all-to-all of self-attention) instead of its own output buffer.
// Unit u = b * H + h (batch entry b, head h) lives on rank u / U; rank r's region holds
// full[3][U][L][128] bf16 (q, k, v of its units for all L = P * Lp tokens) at full_off and the
// arrival flags u32[P] at flag_off. Disabled when P == 0.
constexpr int kXchgMaxPeers = 8;
struct XchgParams {
  unsigned char* base[kXchgMaxPeers];  // every rank's exchange region, as mapped in this process
  long long full_off;
  long long flag_off;
  unsigned int* done_ctr;  // this rank's CTA completion counter (zero between launches)
  unsigned int epoch;      // published into flags[rank] of every region when all CTAs are done
  int P, rank, B, Lp, H, U, L;
};

struct EpiParams {
  const float* vec;  // per-column bias / shift term [N], nullable
  LnFold ln;
  int act;  // kEpiAct: 0 = identity, 1 = tanh-GELU
  // kEpiAct: per-row mean of squares of the bf16 output over each 128-column block of the
  // leading ss_cols columns -> ss_part[row * ss_ld + block] (the RMSNorm partials), nullable
  float* ss_part;
  int ss_ld;
  int ss_cols;
  // residual epilogues
  const float* gate_a;  // [N], nullable (no gate)
  const float* gate_b;  // [batches, gate_b_stride], nullable; gate = gate_a + gate_b[batch]
  int gate_b_stride;
  int rows_per_batch;  // rows of one batch entry along M (per-batch gate rows)
  float* stats_out;    // [M, ceil(N/256), 2], nullable
  void* x_out;         // bf16 copy of the result (long-K variant: direct stores)
  int ldx;
  int has_out_map;
  int has_x_map;
  NormParams norm;  // kEpiNorm only
  XchgParams xchg;  // kEpiNorm only
};

// In-place full-width RMSNorm (+ RoPE) of the leading column groups of a bf16 matrix from
// per-128-column mean-square partials (aux.cu). RoPE tables are token-major: entry
// (token, pair) at token * rope_ld + pair; row r is token r % rows_per_batch + token_offset.
int launch_rms_rope_apply(void* x, int ldx, int M, const float* part, int part_ld, int groups, int width,
                          const float* w0, const float* w1, float eps, int rope_groups, const float* rope_cos,
                          const float* rope_sin, int rope_ld, int rows_per_batch, int token_offset, void* stream);

// Device address of the library's error record {code, site, block, extra} on the current
// device (defined with the GEMM kernels), and the host copy of the device-side wait limit.
int error_record_ptr(unsigned int** out);
unsigned long long wait_limit_ns();

}  // namespace wdit
