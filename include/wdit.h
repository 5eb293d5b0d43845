/*
 * wdit.h - C ABI of the B200 (sm_100a) kernels for the non-attention half of the
 * Wan2.1 DiT block (library: coda-wan-dit_b200/libwdit.so).
 *
 * Conventions
 *   - Plain device pointers, element counts / leading dimensions in ELEMENTS, and a
 *     cudaStream_t passed as `void* stream` (NULL = legacy default stream).
 *   - Matrices are row-major. GEMM operand B is the nn.Linear weight [N, K] (K contiguous),
 *     i.e. the reference's `b_kn` (K, N) argument seen as a transposed view.
 *   - bf16 tensors are `void*` (2-byte elements), fp32 tensors `float*`.
 *   - Nothing here allocates device memory: the caller owns every buffer, including the
 *     scratch workspace of wdit_gemm_norm (size from wdit_gemm_norm_workspace_bytes).
 *   - Return value: 0 on success, a WDIT_ERR_* code otherwise (launch errors are
 *     WDIT_ERR_CUDA_BASE + cudaError_t). Asynchronous device-side failures (a bounded
 *     wait that ran out) are recorded on the device and read with wdit_read_error.
 *   - Alignment: every pointer 16-byte aligned; leading dimensions a multiple of 16 bytes.
 *   - N must be a multiple of 64 and K a multiple of 8 for the GEMMs; M is arbitrary.
 *   - Zero rows (M = 0, or rows / N = 0 where those count the rows) is a no-op that returns
 *     WDIT_OK before any pointer is looked at (an empty tensor may have a null data pointer).
 *
 * Each entry point names the reference (Owen718/CODA-Wan-DiT) interface it replaces.
 */
#ifndef WDIT_H_
#define WDIT_H_

#ifdef __cplusplus
extern "C" {
#endif

#define WDIT_OK 0
#define WDIT_ERR_ARG 1        /* null pointer or inconsistent argument */
#define WDIT_ERR_SHAPE 2      /* unsupported shape */
#define WDIT_ERR_ALIGN 3      /* pointer / stride alignment */
#define WDIT_ERR_ALIAS 4      /* partially overlapping in-place buffers */
#define WDIT_ERR_WORKSPACE 5  /* workspace missing or too small */
#define WDIT_ERR_TMAP 6       /* cuTensorMapEncodeTiled rejected a descriptor */
#define WDIT_ERR_DRIVER 7     /* driver entry point unavailable */
#define WDIT_ERR_SCRATCH_LIMIT 8 /* problem needs more than the static scratch of wdit_gemm_norm_static */

/* Size of the fixed device scratch array used by wdit_gemm_norm_static (per GPU). */
#define WDIT_STATIC_SCRATCH_BYTES (4ll << 20)
#define WDIT_ERR_CUDA_BASE 1000

/* ---- runtime / diagnostics (no reference counterpart; the reference uses Python asserts) ---- */

/* Number of SMs of the current device (the persistent grid size). */
int wdit_num_sms(void);

/* Run the tensor-bound GEMMs (wdit_gemm_act, wdit_gemm_residual with K >= 4096) on CTA pairs
 * (tcgen05 cta_group::2, 256 x 256 tiles) when M > 256: 1 = on (default), 0 = one CTA per
 * 128 x 256 tile. Process-wide; returns the previous setting. Results are identical. */
int wdit_set_cta_pair(int enable);

/* Make `device` current for this library's CUDA runtime in the calling thread (the library
 * links its own runtime; callers keep it equal to their framework's current device). */
int wdit_set_device(int device);

/* Width (columns) of one LayerNorm-statistics partial written by wdit_gemm_residual. */
int wdit_stats_tile_width(void);

/* Upper bound, in nanoseconds, of every device-side wait (default 2 s). */
int wdit_set_wait_limit_ns(unsigned long long ns);

/* Failure-detection self-test: a one-thread kernel waits (bounded by the wait limit) for
 * *flag to become nonzero; if nothing sets it, the wait gives up and records
 * {0x7117 (timeout), 8 (self-test site)} in the error record, leaving the context usable. */
int wdit_wait_selftest(const unsigned int* flag, void* stream);

/* Synchronizes the device and copies the device error record
 * {code, site, block, extra} into out4 (all zero = no error); clear != 0 resets it. */
int wdit_read_error(unsigned int* out4, int clear);

/* ---- fused GEMMs ---- */

/*
 * out[M,N] (bf16) = act( LN(A . B^T) + vec ),   act: 0 identity, 1 tanh-GELU.
 * LN is the absorbed adaLN LayerNorm: rstd_m * (acc - mu_m * ln_csum[n]) where (mu, rstd) of
 * row m are merged from ln_stats[m, 0..ln_stats_tiles-1] = (mean, M2) over ln_stats_width
 * columns each (as written by wdit_gemm_residual / wdit_ln_stats); ln_csum = NULL disables it.
 * ms_out (nullable): ms_out[m * ms_ld + j] = mean over the 128 columns [128j, 128j+128) of
 * bf16(out)^2 for the leading ms_cols columns (ms_cols % 128 == 0), the RMSNorm partials.
 * Replaces: coda_wan/wan_coda_kernels.py:120-152 linear_bias_gelu_fixed (EVTGELUBias :84-105)
 * together with the LN+modulate kernel it consumes (:35-81, removed by the fold); with ms_out,
 * :192-230 qk_linear_bias_partial_rms (EVTColBlockReductionStore with the mean-square op).
 */
int wdit_gemm_act(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                  const float* vec, int act, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                  int ln_stats_width, float ln_eps, float* ms_out, int ms_ld, int ms_cols, void* stream,
                  int max_ctas);

/*
 * out[M,N] (fp32) = C + (A . B^T + bias) * gate,  gate[m, n] = gate_a[n] + gate_b[batch(m), n]
 * (gate_a = NULL: no gate, out = C + A . B^T + bias). batch(m) = m / rows_per_batch.
 * out may alias C exactly (in-place residual update). Optional side outputs:
 * x_bf16_out[M,N] = bf16(out), stats_out[M, ceil(N/256), 2] = per-256-column (mean, M2) of out.
 * Replaces: coda_wan/wan_gate_residual_coda.py:192-242 linear_gate_bias_residual_fixed and
 * :99-135 linear_bias_residual_fixed.
 */
int wdit_gemm_residual(const void* A, int lda, const void* B, int ldb, const float* C, int ldc, float* out, int ldo,
                       int M, int N, int K, const float* bias, const float* gate_a, const float* gate_b,
                       int gate_b_stride, int rows_per_batch, void* x_bf16_out, int ldx, float* stats_out,
                       void* stream, int max_ctas);

/* Workspace bytes wdit_gemm_norm needs: the RMSNorm partials, M x norm_groups * norm_width / 128
 * fp32 (rounded up to 256 bytes). Contents need no initialization. */
long long wdit_gemm_norm_workspace_bytes(int M, int N, int norm_groups, int norm_width);

/*
 * out[M,N] (bf16): y = LN(A . B^T) + vec, rounded to bf16; columns [g*W, (g+1)*W) for
 * g < norm_groups (W % 128 == 0) get the full-width WanRMSNorm
 * bf16(bf16(y * rsqrt(mean_W(y^2) + eps)) * w_g), and for g < rope_groups the interleaved-pair
 * 3D RoPE of 128-column heads with the token-major tables rope_cos/sin[token * rope_ld + pair]
 * (pair < 64, rope_ld >= 64, token = m % rows_per_batch + token_offset; the tables must hold
 * rows_per_batch + token_offset tokens). Remaining columns are stored as bf16(y).
 * QKV: norm_groups 2, rope_groups 2; cross-Q: 1, 0; cross-KV: 1, 0.
 * Two launches on `stream`: the GEMM (bf16 y plus the mean-square partials, in the workspace)
 * and an in-place RMSNorm / RoPE pass over the normalized groups.
 * Replaces: coda_wan/wan_coda_kernels.py:355-368 qk_coda_rms_rope (= :192-230
 * qk_linear_bias_partial_rms + :313-352 qk_rms_rope_from_partials), the V projection at
 * coda_wan/run_wan_coda.py:158, and :371-411 rmsnorm_fused applied to cross-attention q / k.
 */
int wdit_gemm_norm(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                   const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                   int ln_stats_width, float ln_eps, int norm_groups, int norm_width, const float* norm_w0,
                   const float* norm_w1, float norm_eps, int rope_groups, const float* rope_cos, const float* rope_sin,
                   int rope_ld, int rows_per_batch, int token_offset, void* workspace, long long workspace_bytes,
                   void* stream, int max_ctas);

/*
 * The result of wdit_gemm_norm in ONE launch and without a workspace: the GEMM's epilogue
 * applies the full-width RMSNorm and RoPE itself. Each CTA pair owns whole (row block, group)
 * units of norm_width / 256 output tiles, sums each row's squares of the bf16 output over the
 * unit, and after the unit's last tile normalizes / rotates the unit's columns in place (from
 * L2) while its tensor cores start the next unit. Requires norm_groups >= 1 and
 * norm_width % 256 == 0 (else WDIT_ERR_ARG / WDIT_ERR_SHAPE; wdit_gemm_norm takes any
 * multiple of 128). Same arguments and arithmetic as wdit_gemm_norm otherwise; the mean square
 * is summed in another order, so results can differ from wdit_gemm_norm's by a bf16 ulp.
 * Replaces: coda_wan/wan_coda_kernels.py:355-368 qk_coda_rms_rope (the Q+K GEMM :192-230 and
 * the RMSNorm / RoPE kernel :313-352 in one), the V projection at coda_wan/run_wan_coda.py:158,
 * and :371-411 rmsnorm_fused applied to the cross-attention q (coda_wan/run_wan_coda.py:177-179).
 */
int wdit_gemm_norm_fused(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                         const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                         int ln_stats_width, float ln_eps, int norm_groups, int norm_width, const float* norm_w0,
                         const float* norm_w1, float norm_eps, int rope_groups, const float* rope_cos,
                         const float* rope_sin, int rope_ld, int rows_per_batch, int token_offset, void* stream,
                         int max_ctas);

/*
 * Token-sharded (Ulysses) QKV with the all-to-all folded into the GEMM: the same math as
 * wdit_gemm_norm_fused with N = 3 D, norm_groups = rope_groups = 2 (q, k) and rows_per_batch = Lp,
 * but q, k (after RMSNorm / RoPE) and v are stored by the kernel straight into the exchange
 * region of the rank that owns each (batch entry, head) unit, and the last CTA to finish
 * writes `epoch` into flags[rank] of every rank's region (system-scope release). Replaces the
 * QKV GEMM of coda_wan/run_wan_coda.py:158 plus the q/k norm kernel of
 * coda_wan/wan_coda_kernels.py:355-368 and the sequence-to-head all-to-all that the
 * reference's sequence-parallel attention does around them.
 *   A [M = batch * Lp, K] is this rank's token shard (Lp tokens per batch entry, rank r holds
 *     global tokens r * Lp .. r * Lp + Lp - 1); B [3 D, K] is the folded QKV weight; D = 128 H,
 *     a multiple of 256; (batch * H) % P == 0, P <= 8.
 *   qk_scratch [M, ld_scratch >= 3 D] bf16 on this GPU holds the pre-norm q, k.
 *   peer_bases[P]: every rank's exchange region as mapped in this process (256-byte aligned).
 *     Region layout from full_off: bf16 [3][U][L][128], U = batch * H / P units, L = P * Lp;
 *     unit u = b * H + h lives on rank u / U. u32 flags[P] at flag_off.
 *   done_ctr: one u32 on this GPU, zero before the first call; the kernel leaves it zero.
 *   rope_cos / rope_sin: global-token tables with at least P * Lp rows.
 * Returns WDIT_ERR_SHAPE / _ALIGN / _ARG for a bad argument (nothing launched).
 */
int wdit_gemm_norm_exchange(const void* A, int lda, const void* B, int ldb, void* qk_scratch, int ld_scratch, int M,
                            int K, const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                            int ln_stats_width, float ln_eps, const float* wq, const float* wk, float eps,
                            const float* rope_cos, const float* rope_sin, int rope_ld, int batch, int Lp, int H,
                            int P, int rank, const void* const* peer_bases, long long full_off, long long flag_off,
                            unsigned int epoch, unsigned int* done_ctr, void* stream, int max_ctas);

/*
 * wdit_gemm_norm without a workspace argument: it allocates nothing and takes no scratch from
 * the caller. No counterpart in the reference (which always allocates through PyTorch); it is
 * for callers that cannot allocate device memory where they issue this GEMM, e.g. code running
 * where allocation is not allowed or with an allocator owned by another runtime.
 * Same arguments and result as wdit_gemm_norm (norm_groups >= 1). The RMSNorm partials live
 * in a fixed array of WDIT_STATIC_SCRATCH_BYTES (4 MiB) per GPU, held for the life of the
 * process; problems needing more (wdit_gemm_norm_workspace_bytes > 4 MiB, e.g. QKV beyond
 * ~43k rows) return WDIT_ERR_SCRATCH_LIMIT. Every call on a device shares that array: calls
 * that overlap on the GPU race. The first call on a device looks the array's address up (with
 * this library's current device, see wdit_set_device); make it before any stream capture.
 */
int wdit_gemm_norm_static(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                          const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                          int ln_stats_width, float ln_eps, int norm_groups, int norm_width, const float* norm_w0,
                          const float* norm_w1, float norm_eps, int rope_groups, const float* rope_cos,
                          const float* rope_sin, int rope_ld, int rows_per_batch, int token_offset, void* stream,
                          int max_ctas);

/* Bytes of the static scratch array of wdit_gemm_norm_static (= WDIT_STATIC_SCRATCH_BYTES). */
long long wdit_static_scratch_bytes(void);

/* ---- memory-bound passes ---- */

/*
 * Row statistics of x[M,D] (x_is_bf16 selects bf16 or fp32 input) in the format of
 * wdit_gemm_residual's stats_out (per-256-column (mean, M2)); optionally writes bf16(x) and
 * fp32(x). The stats pass for the first block, whose input no residual epilogue produced.
 * Replaces: the statistics half of coda_wan/wan_coda_kernels.py:35-56 (_layernorm_modulation_kernel).
 */
int wdit_ln_stats(const void* x, int x_is_bf16, int ldx, int M, int D, float* stats_out, void* x_bf16_out,
                  float* x_f32_out, void* stream);

/*
 * Per-step weight fold of an adaLN LayerNorm into the following Linear W[N,K] (bf16):
 *   mult[k]  = mult_c + mult_a[k] + mult_b[k]       (mult_b nullable)
 *   shift[k] = shift_a[k] + shift_b[k]              (both nullable)
 *   Wf[n,k]  = bf16(W[n,k] * mult[k]),  csum[n] = sum_k Wf[n,k],
 *   vec[n]   = sum_k shift[k] * W[n,k] + bias[n]    (bias nullable)
 * Modulation: mult_c = 1, mult_a = modulation[scale], mult_b = e[scale], shift = modulation[shift] + e[shift].
 * Static norm3 fold: mult_c = 0, mult_a = gamma, shift_a = beta.
 * Replaces: the modulation add at coda_wan/run_wan_coda.py:142 and the (1 + scale) / shift of
 * coda_wan/wan_coda_kernels.py:52-55, moved from the activations to the weight.
 */
int wdit_fold_weight(const void* W, int ldw, int N, int K, float mult_c, const float* mult_a, const float* mult_b,
                     const float* shift_a, const float* shift_b, const float* bias, void* W_out, int ldw_out,
                     float* csum_out, float* vec_out, void* stream);

/*
 * Many wdit_fold_weight calls in one launch (up to 64 per launch; more are split): all of a
 * forward step's adaLN folds (every block's QKV and FFN1 weights and the head) at once, since
 * they depend only on the step's time embedding. Each job has wdit_fold_weight's arguments
 * and checks; the first failing job's status is returned before anything is launched.
 * Replaces: the per-block modulation at coda_wan/run_wan_coda.py:142 and
 * coda_wan/wan_coda_kernels.py:52-55, for all blocks of a step.
 */
typedef struct wdit_fold_job {
  const void* W;
  int ldw;
  int N;
  int K;
  float mult_c;
  const float* mult_a;
  const float* mult_b;
  const float* shift_a;
  const float* shift_b;
  const float* bias;
  void* W_out;
  int ldw_out;
  float* csum_out;
  float* vec_out;
} wdit_fold_job;
int wdit_fold_weight_batch(const wdit_fold_job* jobs, int n_jobs, void* stream);

/*
 * out[M,D] (bf16) = (x - mean) * rsqrt(var + eps) * (1 + scale) + shift, x fp32 or bf16.
 * Replaces: coda_wan/wan_coda_kernels.py:59-81 layernorm_modulation_bf16.
 */
int wdit_layernorm_modulation(const void* x, int x_is_bf16, int ldx, int M, int D, const float* scale,
                              const float* shift, float eps, void* out, int ldo, void* stream);

/*
 * out[M,D] (bf16) = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w), x bf16.
 * Replaces: coda_wan/wan_coda_kernels.py:392-411 rmsnorm_fused.
 */
int wdit_rmsnorm(const void* x, int ldx, int M, int D, const float* w, float eps, void* out, int ldo, void* stream);

/*
 * Patch rows for the patch embedding as a GEMM: latent[C, F, H, W] (bf16, contiguous), patch
 * (pt, ph, pw) with stride = patch; out[rows, Kp] (bf16) row r = the patch of token
 * token_lo + r of the (F/pt, H/ph, W/pw) grid (frame-major), column ((c*pt + kt)*ph + kh)*pw + kw,
 * K = C*pt*ph*pw <= Kp (Kp % 8 == 0); columns past K and tokens past the grid are zero.
 * out . weight.reshape(D, K)^T + bias (wdit_gemm_act, K padded to Kp) is the Conv3d.
 * Replaces: the Conv3d patch embedding of the stock Wan forward the reference calls at
 * coda_wan/run_wan_coda.py:250 (nn.Conv3d with kernel = stride = patch_size).
 */
int wdit_patch_rows(const void* latent, int C, int F, int H, int W, int pt, int ph, int pw, long long token_lo,
                    int rows, int Kp, void* out, void* stream);

/*
 * In-place WanRMSNorm of `layers` column groups of x[M, ldx] (bf16) from the per-128-column
 * mean-square partials that wdit_gemm_act writes (ms_out): group l is columns
 * [l * x_layer_stride, l * x_layer_stride + width) of every row, its partials start at column
 * l * part_layer_stride of part[M, part_ld] and its weight at w + l * w_layer_stride (fp32).
 * Normalizes the cross-attention K of every block after one GEMM projected the text context
 * through all blocks' packed K/V weights. width % 128 == 0; strides in elements.
 * Replaces: coda_wan/wan_coda_kernels.py:371-411 rmsnorm_fused applied to the cross-attention
 * k of each block (coda_wan/run_wan_coda.py:179-182).
 */
int wdit_rms_apply_layers(void* x, int ldx, int M, const float* part, int part_ld, int width, const float* w,
                          float eps, int layers, long long x_layer_stride, int part_layer_stride, int w_layer_stride,
                          void* stream);

/*
 * In-place WanRMSNorm + RoPE of q and k from per-128-column mean-square partials.
 * qk[M, 2D] bf16, partial[M, 2D/128] fp32, wq/wk[D] fp32, cos/sin[M, 64] fp32.
 * Replaces: coda_wan/wan_coda_kernels.py:313-352 qk_rms_rope_from_partials.
 */
int wdit_qk_rms_rope_from_partials(void* qk, int ldqk, const float* partial, int M, int D, const float* wq,
                                   const float* wk, const float* cos_tab, const float* sin_tab, float eps,
                                   void* stream);

/*
 * cos/sin (fp32) of the 3D RoPE for grid (f, h, w), T = f*h*w tokens, from the per-axis complex
 * frequency table freqs[max_pos, 64] (complex128 stored as interleaved fp64 (re, im) pairs);
 * the 64 pairs split [22, 21, 21] between the frame, height and width axes. Layout: token-major
 * [T, 64] (pair_major = 0, the reference's layout, what wdit_gemm_norm and the exchange kernels
 * read) or pair-major [64, T] (pair_major = 1).
 * Replaces: coda_wan/wan_coda_kernels.py:414-430 build_wan_rope_table.
 */
int wdit_rope_table(const double* freqs_ri, int max_pos, int f, int h, int w, int pair_major, float* cos_out,
                    float* sin_out, void* stream);

/* ---- sequence-parallel (Ulysses) regrouping; no reference counterpart (the reference is
 * single-GPU), these serve the token-sharded multi-GPU forward ----
 * Units: u = b*H + h over the B*H (batch, head) pairs, U = B*H/P units per rank, unit u on
 * rank u / U. Rank r owns tokens [r*Lp, (r+1)*Lp) of every batch entry. hd % 8 == 0.
 */

/* send[P][nmat][U][Lp][hd] <- src rows (b*Lp + t), columns (c*H + h)*hd + i, c < nmat. */
int wdit_ulysses_pack(const void* src, int ld, int B, int Lp, int H, int hd, int nmat, int P, void* send,
                      void* stream);

/* dst[nmat][U][P*Lp][hd] <- recv[P][nmat][U][Lp][hd] (full sequence per unit). */
int wdit_seq_gather(const void* recv, int nmat, int U, int P, int Lp, int hd, void* dst, void* stream);

/* send[P][U][Lp][hd] <- o[j*unit_stride + token*tok_stride + i] (attention output per unit). */
int wdit_seq_scatter(const void* o, long long unit_stride, long long tok_stride, int U, int P, int Lp, int hd,
                     void* send, void* stream);

/* dst rows (b*Lp + t), columns h*hd + i <- recv[P][U][Lp][hd]. */
int wdit_ulysses_unpack(const void* recv, int B, int Lp, int H, int hd, int P, void* dst, int ld, void* stream);

/* ---- the same all-to-all as direct NVLink stores into peer GPUs' memory (no reference
 * counterpart). Each rank exposes an exchange region of its own memory (256-byte aligned):
 *   full[2][3][U][L][hd] bf16 at full_off[buf], y[2][B*Lp][ldy] bf16 at y_off[buf],
 *   flags[2][P] u32 at flag_off[x] (zero before first use)
 * mapped into every peer with CUDA IPC; peer_bases[p] = rank p's region as mapped in the
 * calling process (its own region for p == rank). `epoch` counts exchanges from 1 and picks
 * buffer epoch & 1. Each exchange kernel finishes by publishing epoch into flags[x][rank] of
 * every rank (system-scope release); wdit_p2p_wait blocks the stream until all P ranks have
 * published it (bounded by the wait limit; on expiry the error record holds {0x7117, 9,
 * missing rank, epoch}). done_ctr: one zeroed u32 per exchange kernel, private to the rank. */

/* 64-byte IPC handle of the allocation holding ptr, and ptr's offset inside it. */
int wdit_ipc_handle(const void* ptr, void* handle_out, long long* offset_out);
/* Map a peer's allocation (peer access enabled lazily); base of the mapping. */
int wdit_ipc_open(const void* handle, void** base_out);
int wdit_ipc_close(void* base);

/* Exchange 1: qkv[B*Lp, >= 3*H*hd] (QKV GEMM output, q and k not yet normalized), part[B*Lp,
 * part_ld] (its per-128-column mean squares, q blocks then k blocks), q/k RMSNorm weights,
 * token-major RoPE tables indexed by global token (rank*Lp + t). Writes RMSNorm + RoPE(q, k)
 * and v of every head into full[epoch & 1] of the rank owning its unit. hd = 128. */
int wdit_p2p_qkv_exchange(const void* qkv, int ldq, const float* part, int part_ld, const float* wq,
                          const float* wk, float eps, const float* rope_cos, const float* rope_sin, int rope_ld,
                          int B, int Lp, int H, int hd, int P, int rank, const void* const* peer_bases,
                          long long full_off, long long flag_off, unsigned int epoch, unsigned int* done_ctr,
                          void* stream);

/* Exchange 2: attention output o[j*o_unit_stride + g*o_tok_stride + i] of this rank's units
 * (j < U, global token g < P*Lp) -> y[epoch & 1] rows (b*Lp + t), columns h*hd + i of the rank
 * owning token g. */
int wdit_p2p_out_exchange(const void* o, long long o_unit_stride, long long o_tok_stride, int B, int Lp, int H,
                          int hd, int P, int rank, const void* const* peer_bases, long long y_off, int ldy,
                          long long flag_off, unsigned int epoch, unsigned int* done_ctr, void* stream);

/* Stream-ordered bounded wait until flags[0..P) (this rank's flags of one exchange) reach epoch. */
int wdit_p2p_wait(const unsigned int* flags, int P, unsigned int epoch, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WDIT_H_ */
