// Memory-bound passes around the fused GEMMs. One warp per row everywhere; these
// kernels stream HBM and are sized for it (8 warps per block, grid = rows / 8).
//
//   ln_stats_kernel      per-256-column (mean, M2) of the first block's input rows
//                        (+ bf16 / fp32 copies); stats format = wdit_gemm_residual's.
//   fold_weight_kernel   per-step adaLN fold into the next Linear: W' = W * mult[k],
//                        csum[n] = sum_k W'[n,k], vec[n] = sum_k shift[k] W[n,k] + b[n];
//   fold_batch_kernel    the same for up to 64 weights in one launch (a whole forward step).
//   layernorm_mod_kernel reference op coda_wan/wan_coda_kernels.py:35-81.
//   rmsnorm_kernel       reference op coda_wan/wan_coda_kernels.py:371-411.
//   rms_rope_apply_kernel full-width RMSNorm (+ RoPE) from mean-square partials, in place:
//                        the second half of every norm GEMM and the reference op
//                        coda_wan/wan_coda_kernels.py:233-352.
//   rope_table_kernel    reference op coda_wan/wan_coda_kernels.py:414-430.
//   patch_rows_kernel    im2col of the non-overlapping patch embedding (the Conv3d becomes a
//                        GEMM with the bias in its epilogue).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "wdit_internal.h"

namespace wdit {
namespace {

constexpr int kRowsPerBlock = 8;
constexpr int kSeg = 256;  // statistics tile width (= the GEMM's BN)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const void* base, bool is_bf16, size_t idx, float (&v)[8]) {
  if (is_bf16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + idx);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

__device__ __forceinline__ void store8_bf16(void* base, size_t idx, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + idx) = u;
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) ln_stats_kernel(const void* __restrict__ x, int is_bf16, int ldx, int M, int D,
                                                       float* __restrict__ stats, void* __restrict__ xb,
                                                       float* __restrict__ xf) {
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int nseg = (D + kSeg - 1) / kSeg;
  for (int sgi = 0; sgi < nseg; ++sgi) {
    const int c0 = sgi * kSeg + lane * 8;
    const int width = min(kSeg, D - sgi * kSeg);
    const bool ok = c0 < D;
    float v[8];
    if (ok) {
      load8(x, is_bf16 != 0, static_cast<size_t>(row) * ldx + c0, v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[i];
    const float mean = warp_sum(s) / static_cast<float>(width);
    float m2 = 0.f;
    if (ok) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[i] - mean;
        m2 = fmaf(d, d, m2);
      }
    }
    m2 = warp_sum(m2);
    if (lane == 0) {
      *reinterpret_cast<float2*>(stats + (static_cast<size_t>(row) * nseg + sgi) * 2) = make_float2(mean, m2);
    }
    if (ok && xb != nullptr) store8_bf16(xb, static_cast<size_t>(row) * D + c0, v);
    if (ok && xf != nullptr) {
      float4* p = reinterpret_cast<float4*>(xf + static_cast<size_t>(row) * D + c0);
      p[0] = make_float4(v[0], v[1], v[2], v[3]);
      p[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
}

// ---------------------------------------------------------------------------
// Weight fold. One fold job: W[N,K] -> W'[N,K], csum[N], vec[N] (the arguments of wdit_fold_weight).
struct FoldJob {
  const __nv_bfloat16* W;
  const float* ma;
  const float* mb;
  const float* sa;
  const float* sb;
  const float* bias;
  __nv_bfloat16* Wout;
  float* csum;
  float* vec;
  int ldw, N, K, ldo;
  float mult_c;
};

// The job's multiplier / shift vectors into shared memory (2 K floats).
__device__ __forceinline__ void fold_load_vectors(const FoldJob& j, float* sm_m, float* sm_s) {
  for (int k = threadIdx.x; k < j.K; k += blockDim.x) {
    sm_m[k] = j.mult_c + ((j.ma != nullptr ? j.ma[k] : 0.f) + (j.mb != nullptr ? j.mb[k] : 0.f));
    sm_s[k] = (j.sa != nullptr ? j.sa[k] : 0.f) + (j.sb != nullptr ? j.sb[k] : 0.f);
  }
  __syncthreads();
}

// One row chunk of kFoldVec 16-byte vectors per lane (K <= kFoldVec * 256 in one chunk):
// bf16(W m) stored, the column sum and s . W accumulated.
constexpr int kFoldVec = 6;
__device__ __forceinline__ void fold_chunk(const FoldJob& j, const float* sm_m, const float* sm_s, int n, int c0,
                                           const uint4 (&raw)[kFoldVec], float& cs, float& vs) {
#pragma unroll
  for (int u = 0; u < kFoldVec; ++u) {
    const int k0 = c0 + u * 256;
    if (k0 >= j.K) break;
    const float4 m0 = *reinterpret_cast<const float4*>(sm_m + k0);
    const float4 m1 = *reinterpret_cast<const float4*>(sm_m + k0 + 4);
    const float4 s0 = *reinterpret_cast<const float4*>(sm_s + k0);
    const float4 s1 = *reinterpret_cast<const float4*>(sm_s + k0 + 4);
    const float m[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
    const float sh[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[u]);
    float wf[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      wf[2 * i] = __bfloat162float(__float2bfloat16_rn(f.x * m[2 * i]));
      wf[2 * i + 1] = __bfloat162float(__float2bfloat16_rn(f.y * m[2 * i + 1]));
      cs += wf[2 * i] + wf[2 * i + 1];
      vs = fmaf(sh[2 * i], f.x, vs);
      vs = fmaf(sh[2 * i + 1], f.y, vs);
    }
    store8_bf16(j.Wout, static_cast<size_t>(n) * j.ldo + k0, wf);
  }
}

__device__ __forceinline__ void fold_load_chunk(const FoldJob& j, int n, int c0, uint4 (&raw)[kFoldVec]) {
  const __nv_bfloat16* wr = j.W + static_cast<size_t>(n) * j.ldw;
#pragma unroll
  for (int u = 0; u < kFoldVec; ++u) {
    if (c0 + u * 256 < j.K) raw[u] = *reinterpret_cast<const uint4*>(wr + c0 + u * 256);
  }
}

__device__ __forceinline__ void fold_finish_row(const FoldJob& j, int n, float cs, float vs) {
  cs = warp_sum(cs);
  vs = warp_sum(vs);
  if ((threadIdx.x & 31) == 0) {
    j.csum[n] = cs;
    j.vec[n] = vs + (j.bias != nullptr ? j.bias[n] : 0.f);
  }
}

// Rows n = n0 + warp, n0 + warp + n_step, ... below n1, one warp per row streamed in chunks of
// kFoldVec 16-byte vectors per lane (one chunk for K <= 1536), all of a chunk's loads issued
// before the first use.
__device__ __forceinline__ void fold_rows(const FoldJob& j, const float* sm_m, const float* sm_s, int n0, int n1,
                                          int n_step) {
  const int c_lane = (threadIdx.x & 31) * 8;
  for (int n = n0 + (threadIdx.x >> 5); n < n1; n += n_step) {
    float cs = 0.f, vs = 0.f;
    for (int c0 = c_lane; c0 < j.K; c0 += kFoldVec * 256) {
      uint4 raw[kFoldVec];
      fold_load_chunk(j, n, c0, raw);
      fold_chunk(j, sm_m, sm_s, n, c0, raw, cs, vs);
    }
    fold_finish_row(j, n, cs, vs);
  }
}

// Single fold: the multiplier m[k] = mult_c + mult_a[k] + mult_b[k] and shift s[k] = shift_a[k]
// + shift_b[k] are built once per block in shared memory, then the block's warps stream
// whole rows of W (grid-stride), write bf16(W m) and reduce each row's column sum and s . W.
// The per-row vector traffic comes from shared memory, so the kernel moves only W in and W' out.
__global__ void __launch_bounds__(256) fold_weight_kernel(const __grid_constant__ FoldJob job) {
  extern __shared__ float fold_smem[];
  fold_load_vectors(job, fold_smem, fold_smem + job.K);
  fold_rows(job, fold_smem, fold_smem + job.K, blockIdx.x * kRowsPerBlock, job.N, gridDim.x * kRowsPerBlock);
}

// All of a forward step's folds in one launch. Job i owns blocks [first[i], first[i+1]); each
// block folds kFoldRowsPerCta consecutive rows of its job. Up to kMaxFoldJobs jobs per launch
// (the descriptors travel as the kernel parameter, ~6 KB).
constexpr int kMaxFoldJobs = 64;
constexpr int kFoldRowsPerCta = 64;
struct FoldBatch {
  FoldJob job[kMaxFoldJobs];
  int first[kMaxFoldJobs + 1];
  int n;
};

__global__ void __launch_bounds__(256) fold_batch_kernel(const __grid_constant__ FoldBatch b) {
  extern __shared__ float fold_smem[];
  int lo = 0, hi = b.n - 1;  // the job whose block range holds blockIdx.x
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.first[mid] <= static_cast<int>(blockIdx.x)) lo = mid; else hi = mid - 1;
  }
  const FoldJob& job = b.job[lo];
  fold_load_vectors(job, fold_smem, fold_smem + job.K);
  const int n0 = (static_cast<int>(blockIdx.x) - b.first[lo]) * kFoldRowsPerCta;
  fold_rows(job, fold_smem, fold_smem + job.K, n0, min(n0 + kFoldRowsPerCta, job.N), kRowsPerBlock);
}

// ---------------------------------------------------------------------------
// Row-wise two-pass LayerNorm + modulation, the row re-read from L1/L2 between passes.
__global__ void __launch_bounds__(256)
    layernorm_mod_kernel(const void* __restrict__ x, int is_bf16, int ldx, int M, int D,
                         const float* __restrict__ scale, const float* __restrict__ shift, float eps,
                         __nv_bfloat16* __restrict__ out, int ldo) {
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const size_t base = static_cast<size_t>(row) * ldx;
  float s = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float v[8];
    load8(x, is_bf16 != 0, base + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[i];
  }
  const float mean = warp_sum(s) / static_cast<float>(D);
  float q = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float v[8];
    load8(x, is_bf16 != 0, base + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[i] - mean;
      q = fmaf(d, d, q);
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + eps);
  for (int c = lane * 8; c < D; c += 256) {
    float v[8];
    load8(x, is_bf16 != 0, base + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (v[i] - mean) * rstd * (1.0f + scale[c + i]) + shift[c + i];
    store8_bf16(out, static_cast<size_t>(row) * ldo + c, v);
  }
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int M, int D,
                                                      const float* __restrict__ w, float eps,
                                                      __nv_bfloat16* __restrict__ out, int ldo) {
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const size_t base = static_cast<size_t>(row) * ldx;
  float q = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float v[8];
    load8(x, true, base + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) q = fmaf(v[i], v[i], q);
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(D) + eps);
  for (int c = lane * 8; c < D; c += 256) {
    float v[8];
    load8(x, true, base + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float y = __bfloat162float(__float2bfloat16_rn(v[i] * rstd));
      v[i] = y * w[c + i];
    }
    store8_bf16(out, static_cast<size_t>(row) * ldo + c, v);
  }
}

// ---------------------------------------------------------------------------
// One warp per row: full-width RMSNorm of each of the row's `groups` column groups (`width`
// columns each) from per-128-column mean-square partials, then (rope groups) the 3D RoPE
// rotation, in place. Lane l handles the 16-byte vectors at columns l*8 + 256*j; with
// 128-column heads those always hold the rotation pairs 4*(l%16) .. 4*(l%16)+3, so each lane
// fetches its 4 (cos, sin) once per row (two 16-byte loads from the token-major tables, shared
// by q and k). The first kApplyVec vectors of the row are requested before the partials are
// reduced, so one memory latency covers both.
// Arithmetic of coda_wan/wan_coda_kernels.py:233-352 (_qk_rms_rope_kernel): mean square =
// mean of the block partials, y = bf16(bf16(x * rsqrt(ms + eps)) * w), then the rotation
// (y_e cos - y_o sin, y_e sin + y_o cos) in fp32 and one bf16 rounding.
constexpr int kApplyVec = 12;       // 16-byte vectors per lane in flight (2 x 1536 columns)
constexpr int kApplyRowsPerBlock = 4;

__device__ __forceinline__ uint4 ld_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__global__ void __launch_bounds__(32 * kApplyRowsPerBlock)
    rms_rope_apply_kernel(__nv_bfloat16* __restrict__ x, int ldx, int M, const float* __restrict__ part,
                          int part_ld, int groups, int width, const float* __restrict__ w0,
                          const float* __restrict__ w1, float eps, int rope_groups, const float* __restrict__ cs,
                          const float* __restrict__ sn, int rope_ld, int rows_per_batch, int token_offset,
                          long long x_layer_stride, int part_layer_stride, int w_layer_stride) {
  const int row = blockIdx.x * kApplyRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  // Layer blockIdx.y: its own columns of x, partial columns and weights (one layer unless batched).
  x += static_cast<long long>(blockIdx.y) * x_layer_stride;
  part += static_cast<size_t>(blockIdx.y) * part_layer_stride;
  w0 += static_cast<size_t>(blockIdx.y) * w_layer_stride;
  if (w1 != nullptr) w1 += static_cast<size_t>(blockIdx.y) * w_layer_stride;
  const int total = groups * width;
  __nv_bfloat16* base = x + static_cast<size_t>(row) * ldx;
  uint4 raw[kApplyVec];
#pragma unroll
  for (int u = 0; u < kApplyVec; ++u) {
    const int c = lane * 8 + 256 * u;
    if (c < total) raw[u] = ld_v4(base + c);
  }
  const int parts = width / 128;
  const float* pr = part + static_cast<size_t>(row) * part_ld;
  float ms0 = 0.f, ms1 = 0.f;
  for (int j = lane; j < parts; j += 32) {
    ms0 += pr[j];
    if (groups > 1) ms1 += pr[parts + j];
  }
  float4 c4 = make_float4(1.f, 1.f, 1.f, 1.f), s4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (rope_groups > 0) {
    const int b = row / rows_per_batch;
    const size_t tok = static_cast<size_t>(row - b * rows_per_batch + token_offset);
    c4 = __ldg(reinterpret_cast<const float4*>(cs + tok * rope_ld) + (lane & 15));
    s4 = __ldg(reinterpret_cast<const float4*>(sn + tok * rope_ld) + (lane & 15));
  }
  const float rstd0 = rsqrtf(warp_sum(ms0) / static_cast<float>(parts) + eps);
  const float rstd1 = rsqrtf(warp_sum(ms1) / static_cast<float>(parts) + eps);
  const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
  const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
  for (int c0 = 0; c0 < total; c0 += 256 * kApplyVec) {
    if (c0 > 0) {
#pragma unroll
      for (int u = 0; u < kApplyVec; ++u) {
        const int c = c0 + lane * 8 + 256 * u;
        if (c < total) raw[u] = ld_v4(base + c);
      }
    }
#pragma unroll
    for (int u = 0; u < kApplyVec; ++u) {
      const int c = c0 + lane * 8 + 256 * u;
      if (c >= total) break;
      const int g = c >= width ? 1 : 0;
      const int cg = c - g * width;
      const float* w = g == 0 ? w0 : w1;
      const float rstd = g == 0 ? rstd0 : rstd1;
      const float4 wa = __ldg(reinterpret_cast<const float4*>(w + cg));
      const float4 wb = __ldg(reinterpret_cast<const float4*>(w + cg + 4));
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const uint32_t rw[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
      float v[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(rw[i] << 16);
        v[2 * i + 1] = __uint_as_float(rw[i] & 0xFFFF0000u);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float y = __bfloat162float(__float2bfloat16_rn(v[i] * rstd));
        v[i] = __bfloat162float(__float2bfloat16_rn(y * wv[i]));
      }
      if (g < rope_groups) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float e = v[2 * i], o = v[2 * i + 1];
          v[2 * i] = e * cc[i] - o * ss[i];
          v[2 * i + 1] = e * ss[i] + o * cc[i];
        }
      }
      store8_bf16(base, c, v);
    }
  }
}

// ---------------------------------------------------------------------------
// Patch rows of one latent u[C, F, H, W] (bf16) for a non-overlapping patch (pt, ph, pw):
// row r is token t = tok_lo + r of the (F/pt, H/ph, W/pw) grid (frame-major), column
// k = ((c * pt + kt) * ph + kh) * pw + kw holds u[c, f pt + kt, i ph + kh, j pw + kw], i.e. the
// Conv3d weight [D, C, pt, ph, pw] flattened to [D, K] is the GEMM's B operand. Columns K..Kp-1
// and tokens past the grid are zero. One thread per 8 columns (one 16-byte store).
__global__ void __launch_bounds__(256)
    patch_rows_kernel(const __nv_bfloat16* __restrict__ u, int C, int F, int H, int W, int pt, int ph, int pw,
                      long long tok_lo, int rows, int K, int Kp, __nv_bfloat16* __restrict__ out) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int groups = Kp / 8;
  if (idx >= static_cast<long long>(rows) * groups) return;
  const int row = static_cast<int>(idx / groups);
  const int k0 = static_cast<int>(idx - static_cast<long long>(row) * groups) * 8;
  const int Fp = F / pt, Hp = H / ph, Wp = W / pw;
  const long long ntok = static_cast<long long>(Fp) * Hp * Wp;
  const long long t = tok_lo + row;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0.f;
  if (t < ntok) {
    const int f = static_cast<int>(t / (static_cast<long long>(Hp) * Wp));
    const int rem = static_cast<int>(t - static_cast<long long>(f) * Hp * Wp);
    const int hi = rem / Wp, wi = rem - (rem / Wp) * Wp;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = k0 + i;
      if (k < K) {
        const int kw = k % pw, kh = (k / pw) % ph, kt = (k / (pw * ph)) % pt, c = k / (pw * ph * pt);
        const size_t src = ((static_cast<size_t>(c) * F + f * pt + kt) * H + hi * ph + kh) * W + wi * pw + kw;
        v[i] = __bfloat162float(u[src]);
      }
    }
  }
  store8_bf16(out, static_cast<size_t>(row) * Kp + k0, v);
}

// ---------------------------------------------------------------------------
__global__ void rope_table_kernel(const double* __restrict__ freqs_ri, int max_pos, int f, int h, int w,
                                  int pair_major, float* __restrict__ cos_out, float* __restrict__ sin_out) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(f) * h * w * 64;
  if (idx >= total) return;
  const int pair = static_cast<int>(idx & 63);
  const long long tok = idx >> 6;
  const int wi = static_cast<int>(tok % w);
  const int hi = static_cast<int>((tok / w) % h);
  const int fi = static_cast<int>(tok / (static_cast<long long>(w) * h));
  // Column split [22, 21, 21]: frame, height, width (head_dim 128 -> 44/42/42 dims).
  const int pos = pair < 22 ? fi : (pair < 43 ? hi : wi);
  const double re = freqs_ri[(static_cast<size_t>(pos) * 64 + pair) * 2];
  const double im = freqs_ri[(static_cast<size_t>(pos) * 64 + pair) * 2 + 1];
  const long long o = pair_major ? static_cast<long long>(pair) * (total >> 6) + tok : idx;
  cos_out[o] = static_cast<float>(re);
  sin_out[o] = static_cast<float>(im);
}

inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WDIT_OK : WDIT_ERR_CUDA_BASE + static_cast<int>(e);
}

inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline unsigned row_blocks(int rows) { return static_cast<unsigned>((rows + kRowsPerBlock - 1) / kRowsPerBlock); }

}  // namespace

int launch_rms_rope_apply(void* x, int ldx, int M, const float* part, int part_ld, int groups, int width,
                          const float* w0, const float* w1, float eps, int rope_groups, const float* rope_cos,
                          const float* rope_sin, int rope_ld, int rows_per_batch, int token_offset, void* stream) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (x == nullptr || part == nullptr || w0 == nullptr || (groups > 1 && w1 == nullptr)) return WDIT_ERR_ARG;
  if (M <= 0 || groups < 1 || groups > 2 || width <= 0 || width % 128 != 0 || ldx < groups * width) return WDIT_ERR_SHAPE;
  if (part_ld < groups * (width / 128)) return WDIT_ERR_SHAPE;
  if (!a16(x) || ldx % 8 != 0 || !a16(w0) || (w1 && !a16(w1))) return WDIT_ERR_ALIGN;
  if (rope_groups > 0) {
    if (rope_cos == nullptr || rope_sin == nullptr || rows_per_batch <= 0 || token_offset < 0) return WDIT_ERR_ARG;
    if (rope_ld < 64) return WDIT_ERR_SHAPE;
    if (!a16(rope_cos) || !a16(rope_sin) || rope_ld % 4 != 0) return WDIT_ERR_ALIGN;
  }
  const unsigned blocks = static_cast<unsigned>((M + kApplyRowsPerBlock - 1) / kApplyRowsPerBlock);
  rms_rope_apply_kernel<<<blocks, 32 * kApplyRowsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<__nv_bfloat16*>(x), ldx, M, part, part_ld, groups, width, w0, w1, eps, rope_groups, rope_cos,
      rope_sin, rope_ld, rows_per_batch, token_offset, 0ll, 0, 0);
  return launch_status();
}

int launch_rms_apply_layers(void* x, int ldx, int M, const float* part, int part_ld, int width, const float* w,
                            float eps, int layers, long long x_layer_stride, int part_layer_stride, int w_layer_stride,
                            void* stream) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (x == nullptr || part == nullptr || w == nullptr) return WDIT_ERR_ARG;
  if (M <= 0 || width <= 0 || width % 128 != 0 || layers < 1 || layers > 65535) return WDIT_ERR_SHAPE;
  if (x_layer_stride < 0 || part_layer_stride < 0 || w_layer_stride < 0) return WDIT_ERR_SHAPE;
  // The last layer's columns, partials and weights stay inside the row / weight table.
  if (static_cast<long long>(layers - 1) * x_layer_stride + width > ldx) return WDIT_ERR_SHAPE;
  if (static_cast<long long>(layers - 1) * part_layer_stride + width / 128 > part_ld) return WDIT_ERR_SHAPE;
  if (!a16(x) || ldx % 8 != 0 || x_layer_stride % 8 != 0 || !a16(w) || w_layer_stride % 4 != 0) return WDIT_ERR_ALIGN;
  const dim3 grid(static_cast<unsigned>((M + kApplyRowsPerBlock - 1) / kApplyRowsPerBlock), static_cast<unsigned>(layers));
  rms_rope_apply_kernel<<<grid, 32 * kApplyRowsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<__nv_bfloat16*>(x), ldx, M, part, part_ld, 1, width, w, nullptr, eps, 0, nullptr, nullptr, 0, 1,
      0, x_layer_stride, part_layer_stride, w_layer_stride);
  return launch_status();
}

}  // namespace wdit

using namespace wdit;

namespace {
int fold_job_check(const wdit_fold_job& j) {
  if (j.N == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (j.W == nullptr || j.W_out == nullptr || j.csum_out == nullptr || j.vec_out == nullptr) return WDIT_ERR_ARG;
  if (j.N <= 0 || j.K <= 0 || j.K % 8 != 0 || j.ldw < j.K || j.ldw_out < j.K) return WDIT_ERR_SHAPE;
  if (!a16(j.W) || !a16(j.W_out) || j.ldw % 8 != 0 || j.ldw_out % 8 != 0) return WDIT_ERR_ALIGN;
  if ((j.mult_a && !a16(j.mult_a)) || (j.mult_b && !a16(j.mult_b)) || (j.shift_a && !a16(j.shift_a)) ||
      (j.shift_b && !a16(j.shift_b)))
    return WDIT_ERR_ALIGN;
  return WDIT_OK;
}

FoldJob fold_job_dev(const wdit_fold_job& j) {
  FoldJob d;
  d.W = reinterpret_cast<const __nv_bfloat16*>(j.W);
  d.ma = j.mult_a;
  d.mb = j.mult_b;
  d.sa = j.shift_a;
  d.sb = j.shift_b;
  d.bias = j.bias;
  d.Wout = reinterpret_cast<__nv_bfloat16*>(j.W_out);
  d.csum = j.csum_out;
  d.vec = j.vec_out;
  d.ldw = j.ldw;
  d.N = j.N;
  d.K = j.K;
  d.ldo = j.ldw_out;
  d.mult_c = j.mult_c;
  return d;
}

// Dynamic shared memory above the 48 KB default (K > 6144) needs the opt-in, once per device.
template <typename Kernel>
void allow_fold_smem(Kernel kernel, size_t smem, bool (&done)[64]) {
  if (smem <= 48 * 1024) return;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[dev & 63]) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    done[dev & 63] = true;
  }
}
}  // namespace


extern "C" {

int wdit_ln_stats(const void* x, int x_is_bf16, int ldx, int M, int D, float* stats_out, void* x_bf16_out,
                  float* x_f32_out, void* stream) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (x == nullptr || stats_out == nullptr) return WDIT_ERR_ARG;
  if (M <= 0 || D <= 0 || D % 8 != 0 || ldx < D) return WDIT_ERR_SHAPE;
  if (!a16(x) || ldx % 8 != 0 || (reinterpret_cast<uintptr_t>(stats_out) & 7) != 0) return WDIT_ERR_ALIGN;
  if ((x_bf16_out && !a16(x_bf16_out)) || (x_f32_out && !a16(x_f32_out))) return WDIT_ERR_ALIGN;
  if (M == 0) return WDIT_OK;
  ln_stats_kernel<<<row_blocks(M), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, x_is_bf16, ldx, M, D, stats_out,
                                                                                 x_bf16_out, x_f32_out);
  return launch_status();
}

int wdit_fold_weight(const void* W, int ldw, int N, int K, float mult_c, const float* mult_a, const float* mult_b,
                     const float* shift_a, const float* shift_b, const float* bias, void* W_out, int ldw_out,
                     float* csum_out, float* vec_out, void* stream) {
  const wdit_fold_job j = {W, ldw, N, K, mult_c, mult_a, mult_b, shift_a, shift_b, bias, W_out, ldw_out, csum_out,
                           vec_out};
  const int rc = fold_job_check(j);
  if (rc || N == 0) return rc;
  const size_t smem = static_cast<size_t>(K) * 2 * sizeof(float);
  static bool attr_set[64] = {};
  allow_fold_smem(fold_weight_kernel, smem, attr_set);
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  unsigned blocks = row_blocks(N);
  if (blocks > static_cast<unsigned>(4 * sms)) blocks = static_cast<unsigned>(4 * sms);
  fold_weight_kernel<<<blocks, 256, smem, static_cast<cudaStream_t>(stream)>>>(fold_job_dev(j));
  return launch_status();
}

int wdit_fold_weight_batch(const wdit_fold_job* jobs, int n_jobs, void* stream) {
  if (n_jobs < 0 || (n_jobs > 0 && jobs == nullptr)) return WDIT_ERR_ARG;
  int max_k = 0;
  for (int i = 0; i < n_jobs; ++i) {
    const int rc = fold_job_check(jobs[i]);
    if (rc) return rc;
    if (jobs[i].N > 0 && jobs[i].K > max_k) max_k = jobs[i].K;
  }
  const size_t smem = static_cast<size_t>(max_k) * 2 * sizeof(float);
  static bool attr_set[64] = {};
  allow_fold_smem(fold_batch_kernel, smem, attr_set);
  for (int j0 = 0; j0 < n_jobs; j0 += kMaxFoldJobs) {
    FoldBatch b;
    b.n = n_jobs - j0 < kMaxFoldJobs ? n_jobs - j0 : kMaxFoldJobs;
    int ctas = 0;
    for (int i = 0; i < b.n; ++i) {
      b.job[i] = fold_job_dev(jobs[j0 + i]);
      b.first[i] = ctas;
      ctas += (jobs[j0 + i].N + kFoldRowsPerCta - 1) / kFoldRowsPerCta;
    }
    b.first[b.n] = ctas;
    if (ctas == 0) continue;  // only empty jobs in this group
    fold_batch_kernel<<<ctas, 256, smem, static_cast<cudaStream_t>(stream)>>>(b);
    const int rc = launch_status();
    if (rc) return rc;
  }
  return WDIT_OK;
}

int wdit_layernorm_modulation(const void* x, int x_is_bf16, int ldx, int M, int D, const float* scale,
                              const float* shift, float eps, void* out, int ldo, void* stream) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (x == nullptr || scale == nullptr || shift == nullptr || out == nullptr) return WDIT_ERR_ARG;
  if (M <= 0 || D <= 0 || D % 8 != 0 || ldx < D || ldo < D) return WDIT_ERR_SHAPE;
  if (!a16(x) || !a16(out) || ldx % 8 != 0 || ldo % 8 != 0) return WDIT_ERR_ALIGN;
  layernorm_mod_kernel<<<row_blocks(M), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_is_bf16, ldx, M, D, scale, shift, eps, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return launch_status();
}

int wdit_rmsnorm(const void* x, int ldx, int M, int D, const float* w, float eps, void* out, int ldo, void* stream) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (x == nullptr || w == nullptr || out == nullptr) return WDIT_ERR_ARG;
  if (M <= 0 || D <= 0 || D % 8 != 0 || ldx < D || ldo < D) return WDIT_ERR_SHAPE;
  if (!a16(x) || !a16(out) || ldx % 8 != 0 || ldo % 8 != 0) return WDIT_ERR_ALIGN;
  rmsnorm_kernel<<<row_blocks(M), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, D, w, eps, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return launch_status();
}

int wdit_qk_rms_rope_from_partials(void* qk, int ldqk, const float* partial, int M, int D, const float* wq,
                                   const float* wk, const float* cos_tab, const float* sin_tab, float eps,
                                   void* stream) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (qk == nullptr || partial == nullptr || wq == nullptr || wk == nullptr || cos_tab == nullptr ||
      sin_tab == nullptr)
    return WDIT_ERR_ARG;
  if (M <= 0 || D <= 0 || D % 128 != 0 || ldqk < 2 * D) return WDIT_ERR_SHAPE;
  // The reference's partials [M, 2 * D/128] (q blocks, then k blocks) and [M, 64] tables
  // indexed by row are this pass's layout with two rope groups.
  return launch_rms_rope_apply(qk, ldqk, M, partial, 2 * (D / 128), 2, D, wq, wk, eps, 2, cos_tab, sin_tab, 64, M, 0,
                               stream);
}

int wdit_rope_table(const double* freqs_ri, int max_pos, int f, int h, int w, int pair_major, float* cos_out,
                    float* sin_out, void* stream) {
  if (freqs_ri == nullptr || cos_out == nullptr || sin_out == nullptr) return WDIT_ERR_ARG;
  if (f <= 0 || h <= 0 || w <= 0 || f > max_pos || h > max_pos || w > max_pos) return WDIT_ERR_SHAPE;
  const long long total = static_cast<long long>(f) * h * w * 64;
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
  rope_table_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(freqs_ri, max_pos, f, h, w, pair_major,
                                                                            cos_out, sin_out);
  return launch_status();
}

int wdit_patch_rows(const void* latent, int C, int F, int H, int W, int pt, int ph, int pw, long long token_lo,
                    int rows, int Kp, void* out, void* stream) {
  if (rows == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (latent == nullptr || out == nullptr) return WDIT_ERR_ARG;
  if (C <= 0 || pt <= 0 || ph <= 0 || pw <= 0 || F < pt || H < ph || W < pw || rows <= 0 || token_lo < 0)
    return WDIT_ERR_SHAPE;
  const int K = C * pt * ph * pw;
  if (Kp < K || Kp % 8 != 0) return WDIT_ERR_SHAPE;
  if (!a16(out)) return WDIT_ERR_ALIGN;
  const long long total = static_cast<long long>(rows) * (Kp / 8);
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
  patch_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(latent), C, F, H, W, pt, ph, pw, token_lo, rows, K, Kp,
      reinterpret_cast<__nv_bfloat16*>(out));
  return launch_status();
}

int wdit_rms_apply_layers(void* x, int ldx, int M, const float* part, int part_ld, int width, const float* w,
                          float eps, int layers, long long x_layer_stride, int part_layer_stride, int w_layer_stride,
                          void* stream) {
  return launch_rms_apply_layers(x, ldx, M, part, part_ld, width, w, eps, layers, x_layer_stride, part_layer_stride,
                                 w_layer_stride, stream);
}

}  // extern "C"
