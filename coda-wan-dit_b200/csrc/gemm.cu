// Persistent warp-specialized tcgen05 GEMM with the Wan block's fused epilogues.
//
//   D[M, N] = A[M, K] . B[N, K]^T      A, B bf16 K-major (B = nn.Linear.weight layout),
//                                       fp32 accumulation in TMEM.
//
// CTA = 10 warps (320 threads), one CTA per SM, grid = the co-resident CTA count, static tile order
// tile -> (m_blk, n_blk) row-major, or in groups of 8 row blocks for a large B (tile_coords):
//   warp 0     TMA producer: A (128x64) and B (256x64) tiles, 128-byte swizzle,
//              STAGES-deep shared-memory ring (full/empty mbarriers).
//   warp 1     TMEM allocator (512 columns = two 128x256 fp32 accumulators) and
//              single-thread tcgen05.mma issuer (M=128, N=256, K=16 per instruction).
//   warps 2-9  epilogue: tcgen05.ld (thread = one accumulator row; warps 2-5 take columns
//              0-127 of the tile, warps 6-9 columns 128-255), fused math, swizzled
//              shared-memory staging, TMA stores. The residual epilogues use warps 2-5.
// The accumulator is double buffered, so the epilogue of tile i overlaps the mainloop of
// tile i+1.
//
// CTA pairs (PAIR = true, cluster of 2): the tensor-bound variants run 256 x 256 tiles with
// tcgen05 cta_group::2: each CTA loads its 128 rows of A and one 128-row half of B, the even
// CTA issues M=256 MMAs over both CTAs' shared memory, and each CTA's epilogue drains its
// own 128 accumulator rows. Half the B traffic per CTA, same epilogue.
//
// Epilogue families (one template instance each):
//   kEpiAct            out_bf16 = act( LN(acc) + vec )      FFN1 (tanh-GELU), QKV, cross-Q,
//                      cross-KV, text MLP, head; optionally the per-row mean square of the
//                      bf16 output over each 128-column block (RMSNorm partials, consumed by
//                      the in-place RMSNorm / RoPE pass in aux.cu).
//   kEpiNorm           kEpiAct (identity activation) with the full-width WanRMSNorm (+ 3D RoPE)
//                      of the leading column groups applied in the epilogue: QKV, cross-Q.
//                      One CTA (pair) owns whole (row block, group) units of width/256 tiles,
//                      sums each row's squares over the unit, and after the unit's last tile
//                      normalizes / rotates the unit's columns in place from L2 while the MMA
//                      runs ahead (see norm_pass_rows).
//   kEpiResidual       out_f32 = C + (acc + bias) * gate    self-O (gate), cross-O (no gate),
//   kEpiResidualLongK  (short / long K)                     FFN2 (gate)
//                      and optionally a bf16 copy of out plus per-row (mean, M2) partials
//                      of out over each 256-column tile (the next LayerNorm's statistics).
//
// LN(acc) is the adaLN LayerNorm absorbed into the GEMM (the modulation scale is folded
// into the weight each step):  LN(acc) = rstd * (acc - mu * csum[n]),
// with (mu, rstd) merged from the (mean, M2) partials emitted by the previous residual
// epilogue (Chan's parallel variance merge), and the shift term added through `vec`.
//
// Reference counterparts (Owen718/CODA-Wan-DiT):
//   kEpiAct            coda_wan/wan_coda_kernels.py:84-152 (EVTGELUBias, linear_bias_gelu_fixed)
//                      and :155-230 (Q+K GEMM with mean-square partials)
//   kEpiResidual*      coda_wan/wan_gate_residual_coda.py:75-135, 138-161, 192-242
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "ptx.cuh"
#include "wdit_internal.h"

namespace wdit {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int kThreads = 320;     // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpiThreads = 128;  // one column half (4 warps)
constexpr uint32_t kStgBytes = 8192;       // 128 rows x 32 bf16 output staging tile
constexpr uint32_t kWarpStgBytes = 2048;   // 32 rows x 32 bf16: one warp's staging buffer
constexpr uint32_t kTileABytes = BM * BK * 2;  // 16 KB
constexpr uint32_t kTileBBytes = BN * BK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kTileABytes + kTileBBytes;
// CTA pair (cta_group::2): the pair computes a 256 x 256 tile; each CTA stages its 128 rows
// of A and one 128-row half of B, and holds its 128 accumulator rows in its own TMEM.
constexpr uint32_t kPairStageBytes = kTileABytes + kTileBBytes / 2;  // 32 KB
constexpr int kTmemCols = 2 * BN;  // two accumulator buffers
constexpr int kRasterRows = 8;     // row blocks per rasterization group for a large B (tile_coords)
constexpr long long kRasterBBytes = 64ll << 20;  // B operands above this get grouped rasterization
enum EpiKind { kEpiAct = 0, kEpiResidual = 1, kEpiResidualLongK = 3, kEpiNorm = 4 };

template <int KIND>
struct Cfg;
template <>
struct Cfg<kEpiAct> {
  static constexpr int kStages = 4;
  static constexpr int kPairStages = 6;
  // 8 warps x 2 staging buffers (32 rows x 32 bf16, 64-byte swizzle)
  static constexpr uint32_t kEpiBytes = 8 * 2 * kWarpStgBytes;
  static constexpr int kNumCBuf = 0;
  static constexpr int kEpiArrivals = 2 * kEpiThreads;
};
template <>
struct Cfg<kEpiNorm> {
  static constexpr int kStages = 4;
  static constexpr int kPairStages = 6;
  // kEpiAct's staging + the per-row sums of squares of the two column halves [2][128] fp32
  static constexpr uint32_t kEpiBytes = 8 * 2 * kWarpStgBytes + 2 * BM * 4;
  static constexpr int kNumCBuf = 0;
  static constexpr int kEpiArrivals = 2 * kEpiThreads;
};
// Residual epilogues stream the fp32 residual through a ring of 128-row x 32-column fp32
// tiles (16 KB, 128-byte swizzle): TMA load, in-place update, TMA store. kLookahead chunks
// are requested ahead of the one being processed.
//   short K (self-O, cross-O; HBM-bound): deeper ring, 3 mainloop stages
//   long K  (FFN2; tensor-bound): 4 mainloop stages, shallow ring
template <>
struct Cfg<kEpiResidual> {
  static constexpr int kStages = 3;
  static constexpr int kPairStages = 0;  // HBM-bound: the pair buys nothing
  static constexpr int kHalves = 2;      // both column halves' warps work (latency-bound epilogue)
  static constexpr int kNumCBuf = 4;     // 2 per half
  static constexpr int kLookahead = 1;   // per half
  static constexpr bool kXStaged = true;  // bf16 copy staged (64-byte swizzle) + TMA store
  // ring + one staging tile per half + the halves' row-statistics exchange (128 x 3 floats)
  static constexpr uint32_t kEpiBytes = kNumCBuf * 16384 + 2 * kStgBytes + 128 * 3 * 4;
  static constexpr int kEpiArrivals = kHalves * kEpiThreads;
};
template <>
struct Cfg<kEpiResidualLongK> {
  static constexpr int kStages = 4;
  static constexpr int kPairStages = 6;
  static constexpr int kHalves = 1;
  static constexpr int kNumCBuf = 2;
  static constexpr int kLookahead = 1;
  static constexpr bool kXStaged = false;  // bf16 copy stored from registers
  static constexpr uint32_t kEpiBytes = kNumCBuf * 16384;
  static constexpr int kEpiArrivals = kEpiThreads;
};

template <int KIND>
__host__ __device__ constexpr int num_threads() {
  return kThreads;
}
template <int KIND, bool PAIR>
__host__ __device__ constexpr int num_stages() {
  return PAIR ? Cfg<KIND>::kPairStages : Cfg<KIND>::kStages;
}
template <int KIND, bool PAIR>
constexpr uint32_t smem_bytes() {
  return 1024 /*alignment slack*/ + num_stages<KIND, PAIR>() * (PAIR ? kPairStageBytes : kStageBytes) +
         Cfg<KIND>::kEpiBytes + 256 /*barriers + tmem slot*/;
}
static_assert(smem_bytes<kEpiAct, true>() <= 232448 && smem_bytes<kEpiResidualLongK, true>() <= 232448 &&
                  smem_bytes<kEpiResidual, false>() <= 232448 && smem_bytes<kEpiNorm, true>() <= 232448 &&
                  smem_bytes<kEpiNorm, false>() <= 232448,
              "configuration exceeds the 227 KB shared-memory limit");

// ---------------------------------------------------------------------------
// Epilogue helpers
// ---------------------------------------------------------------------------
// tanh-GELU of two columns: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), constants as in
// coda_wan/wan_coda_kernels.py:100-101, factored as z = x (k + k c x^2), out = h + h tanh(z)
// with h = x / 2, in packed f32x2 arithmetic.
__device__ __forceinline__ void gelu_tanh2(float& a, float& b) {
  constexpr float kK = 0.7978845608028654f;
  constexpr float kKC = 0.7978845608028654f * 0.044715f;
  const uint64_t x = f2_pack(a, b);
  const uint64_t z = fmul2(x, ffma2(fmul2(x, x), f2_pack(kKC, kKC), f2_pack(kK, kK)));
  float z0, z1;
  f2_unpack(z, z0, z1);
  const uint64_t h = fmul2(x, f2_pack(0.5f, 0.5f));
  f2_unpack(ffma2(h, f2_pack(tanh_approx(z0), tanh_approx(z1)), h), a, b);
}

// Merge per-tile (mean, M2) partials of one row into (mu, rstd). The partials are fetched
// four at a time so their load latencies overlap.
__device__ __forceinline__ void ln_row_stats(const LnFold& ln, int row, float& mu, float& rstd) {
  const float2* st = reinterpret_cast<const float2*>(ln.stats) + static_cast<size_t>(row) * ln.stats_tiles;
  float n = 0.f, mean = 0.f, m2 = 0.f;
  for (int t0 = 0; t0 < ln.stats_tiles; t0 += 4) {
    float2 pm[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) pm[u] = t0 + u < ln.stats_tiles ? st[t0 + u] : make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u;
      if (t >= ln.stats_tiles) break;
      const int rem = ln.row_len - t * ln.stats_width;
      const float nt = static_cast<float>(rem < ln.stats_width ? rem : ln.stats_width);
      const float tot = n + nt;
      const float delta = pm[u].x - mean;
      mean += delta * (nt / tot);
      m2 += pm[u].y + delta * delta * (n * nt / tot);
      n = tot;
    }
  }
  mu = mean;
  rstd = rsqrtf(m2 / static_cast<float>(ln.row_len) + ln.eps);
}

// In-place WanRMSNorm (+ RoPE) of rows [r0, r1) of one finished (row block, group) unit of the
// norm GEMM, run by the eight epilogue warps: warp ew takes rows r0 + ew, r0 + ew + 8, ...,
// kPassRows at a time (all their loads in flight together). Per row, lane l holds the 16-byte
// vectors at columns 8 l + 256 u of the group, so its rotary pairs are the same four,
// (l % 16) * 4 .. + 3, in every head (one float4 of cos and one of sin per row). The unit's bf16
// GEMM output was stored by TMA and is read back from L2 (ld.global.cg). Arithmetic of
// coda_wan/wan_coda_kernels.py:233-352 (_qk_rms_rope_kernel) and :371-411 (_rmsnorm_kernel):
// rstd = rsqrt(mean(y^2) + eps) over the group's full width (y = the bf16 GEMM output),
// z = bf16(bf16(y rstd) w), then (z_e cos - z_o sin, z_e sin + z_o cos) in fp32, one rounding;
// two columns per packed f32x2 instruction.
constexpr int kPassVec = 6;   // 16-byte vectors per lane and row in flight (one 1536-column row)
constexpr int kPassRows = 2;  // rows per warp in flight

// bf16 rounding of a packed pair, back to a packed fp32 pair
__device__ __forceinline__ uint64_t bf16_round2(uint64_t x) {
  float a, b;
  f2_unpack(x, a, b);
  const float2 r = unpack_bf16x2(pack_bf16x2(a, b));
  return f2_pack(r.x, r.y);
}

// Address in the exchange region of the rank owning unit (b, head of column c) for matrix mat
// (0 q, 1 k, 2 v), global token gtok, column c of the matrix (c % 128 inside the head).
__device__ __forceinline__ unsigned char* xchg_addr(const XchgParams& xc, int mat, int b, int gtok, int c) {
  const int h = c >> 7;
  const int u = b * xc.H + h;
  const int pr = u / xc.U;
  const int ul = u - pr * xc.U;
  return xc.base[pr] + xc.full_off +
         ((((static_cast<long long>(mat) * xc.U + ul) * xc.L + gtok) * 128 + (c & 127)) * 2);
}

__device__ __forceinline__ void norm_pass_rows(const NormParams& np, const XchgParams& xc, const float* ss_x,
                                               int m_blk, int g, int M, int rows_per_batch, int ew, int lane,
                                               int r0, int r1) {
  const float* wg = g == 0 ? np.w0 : np.w1;
  const bool rope = g < np.rope_groups;
  const bool remote = xc.P > 0;  // results go to the owners' exchange regions, not in place
  const int rend = min(r1, M - m_blk * BM);  // rows past M hold no data
#pragma unroll 1
  for (int rr0 = r0 + ew; rr0 < rend; rr0 += 8 * kPassRows) {
    uint64_t rstd2[kPassRows];
    uint64_t cs2[kPassRows][4], sc2[kPassRows][4];  // (cos, sin) and (sin, cos) of the lane's pairs
    __nv_bfloat16* base[kPassRows];
    int xb[kPassRows], xtok[kPassRows];  // remote: batch entry and global token of the row
#pragma unroll
    for (int j = 0; j < kPassRows; ++j) {
      const int rr = min(rr0 + 8 * j, rend - 1);  // a clamped duplicate row is computed, not stored
      const int row = m_blk * BM + rr;
      const float rstd = rsqrtf((ss_x[rr] + ss_x[BM + rr]) * np.inv_width + np.eps);
      rstd2[j] = f2_pack(rstd, rstd);
      float cc[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
      if (rope) {
        const size_t tok = static_cast<size_t>(row % rows_per_batch + np.token_offset);
        const float4 c4 = __ldg(reinterpret_cast<const float4*>(np.cos + tok * np.rope_ld) + (lane & 15));
        const float4 s4 = __ldg(reinterpret_cast<const float4*>(np.sin + tok * np.rope_ld) + (lane & 15));
        cc[0] = c4.x; cc[1] = c4.y; cc[2] = c4.z; cc[3] = c4.w;
        sn[0] = s4.x; sn[1] = s4.y; sn[2] = s4.z; sn[3] = s4.w;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        cs2[j][i] = f2_pack(cc[i], sn[i]);
        sc2[j][i] = f2_pack(sn[i], cc[i]);
      }
      base[j] = reinterpret_cast<__nv_bfloat16*>(np.out) + static_cast<size_t>(row) * np.ldo +
                static_cast<size_t>(g) * np.width;
      xb[j] = remote ? row / xc.Lp : 0;
      xtok[j] = remote ? xc.rank * xc.Lp + (row - xb[j] * xc.Lp) : 0;
    }
#pragma unroll 1
    for (int c0 = 0; c0 < np.width; c0 += 256 * kPassVec) {
      uint4 raw[kPassRows][kPassVec];
#pragma unroll
      for (int j = 0; j < kPassRows; ++j) {
#pragma unroll
        for (int u = 0; u < kPassVec; ++u) {
          const int c = c0 + 256 * u + lane * 8;
          if (c < np.width) raw[j][u] = ld_global_cg_v4(base[j] + c);
        }
      }
#pragma unroll
      for (int u = 0; u < kPassVec; ++u) {
        const int c = c0 + 256 * u + lane * 8;
        if (c >= np.width) break;
        const float4 wa = __ldg(reinterpret_cast<const float4*>(wg + c));
        const float4 wb = __ldg(reinterpret_cast<const float4*>(wg + c + 4));
        const uint64_t w2[4] = {f2_pack(wa.x, wa.y), f2_pack(wa.z, wa.w), f2_pack(wb.x, wb.y), f2_pack(wb.z, wb.w)};
#pragma unroll
        for (int j = 0; j < kPassRows; ++j) {
          if (rr0 + 8 * j >= rend) break;
          const uint32_t rw[4] = {raw[j][u].x, raw[j][u].y, raw[j][u].z, raw[j][u].w};
          uint32_t outw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 x = unpack_bf16x2(rw[i]);
            const uint64_t y = bf16_round2(fmul2(f2_pack(x.x, x.y), rstd2[j]));
            uint64_t z = bf16_round2(fmul2(y, w2[i]));
            if (rope) {
              float e, o;
              f2_unpack(z, e, o);
              // (e cos - o sin, e sin + o cos) = (e, e) * (cos, sin) + (-o, o) * (sin, cos)
              z = ffma2(f2_pack(-o, o), sc2[j][i], fmul2(f2_pack(e, e), cs2[j][i]));
            }
            float a, b;
            f2_unpack(z, a, b);
            outw[i] = pack_bf16x2(a, b);
          }
          void* dst = remote ? static_cast<void*>(xchg_addr(xc, g, xb[j], xtok[j], c))
                             : static_cast<void*>(base[j] + c);
          st_global_v4(dst, outw[0], outw[1], outw[2], outw[3]);
        }
      }
    }
  }
}

// Prefetch rows [r0, r1) of a finished unit's group columns into L2 (one 128-byte line per lane
// and step), so that a later norm_pass_rows over them finds them there.
__device__ __forceinline__ void norm_prefetch_rows(const NormParams& np, int m_blk, int g, int M, int ew, int lane,
                                                   int r0, int r1) {
  const int rend = min(r1, M - m_blk * BM);
  const int row_bytes = np.width * 2;
  for (int rr = r0 + ew; rr < rend; rr += 8) {
    const char* base = reinterpret_cast<const char*>(np.out) +
                       (static_cast<size_t>(m_blk * BM + rr) * np.ldo + static_cast<size_t>(g) * np.width) * 2;
    for (int off = lane * 128; off < row_bytes; off += 32 * 128) prefetch_l2(base + off);
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int KIND, bool PAIR>
__global__ void __launch_bounds__(num_threads<KIND>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmC,
                const __grid_constant__ CUtensorMap tmX, const GemmShape s, const EpiParams p) {
  constexpr int STAGES = num_stages<KIND, PAIR>();
  static_assert(STAGES > 0, "no pair variant for this epilogue");
  constexpr uint32_t SB = PAIR ? kPairStageBytes : kStageBytes;
  // Accumulator-release arrivals per CTA: one per thread, or (pair) one per warp so that the
  // peer CTA sends few remote arrivals to the leader.
  constexpr int kTemptyCount = PAIR ? 2 * (Cfg<KIND>::kEpiArrivals / 32) : Cfg<KIND>::kEpiArrivals;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stage_base = smem;
  uint8_t* epi_base = smem + STAGES * SB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_base + Cfg<KIND>::kEpiBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* cload_bar = tempty_bar + 2;  // kNumCBuf entries (residual only)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cload_bar + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Tile schedule. 1-CTA: CTA b takes tiles t = b, b + grid, ... (tile_coords maps t to a row
  // block and an N block). Pair: s.tiles counts 256-row pair tiles; pair c = blockIdx / 2 takes
  // t = c, c + grid/2, ... and CTA rank r of the pair owns 128-row block 2 mq + r of pair row mq.
  const int cta_rank = PAIR ? static_cast<int>(cluster_ctarank()) : 0;
  const int t_first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int t_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  // Rasterization: tiles run in groups of s.raster_rows row blocks (256-row pair blocks for
  // pairs), row-minor inside a group. raster_rows = 1 is the plain row-major order (a row
  // block's N blocks in turn: its A rows stay hot while the whole B is L2-resident). For a B
  // larger than L2 (the 14B layers: 142-157 MB) the host picks groups of kRasterRows: the tiles
  // in flight then share a few row blocks of A and a few column blocks of B, and B is read from
  // HBM about once per group instead of once per row block.
  auto tile_coords = [&](int t, int& m_blk, int& n_blk) {
    const int mg = PAIR ? (s.m_blocks + 1) / 2 : s.m_blocks;
    const int per_group = s.raster_rows * s.n_blocks;
    const int grp = t / per_group;
    const int first = grp * s.raster_rows;
    const int gm = min(s.raster_rows, mg - first);
    const int r = t - grp * per_group;
    n_blk = r / gm;
    const int mq = first + (r - n_blk * gm);
    m_blk = PAIR ? 2 * mq + cta_rank : mq;
  };
  // This CTA's (pair's) tile sequence i = 0 .. my_count - 1 -> (m_blk, n_blk, upos).
  // Plain kinds: tile t_first + i * t_step. kEpiNorm: units u = t_first + j * t_step, unit u =
  // (row group u / norm_groups, normalized group g = u % norm_groups): the group's unit_tiles
  // tiles (upos = 0 .. unit_tiles - 1), then group g's share of the row group's plain tiles
  // (upos = -1; the plain tiles of a row group are split evenly over its normalized groups, a
  // remainder going to the groups (g + row group) % norm_groups < remainder), so that every
  // tile of a row group runs at about the same time (its A rows are read from HBM once) and the
  // normalize pass of a unit runs while its plain tiles are computed.
  int my_count = 0;
  int seq_units = 0;
  const int ng = KIND == kEpiNorm ? s.norm_groups : 1;
  const int vbase = KIND == kEpiNorm ? s.plain_nblocks / ng : 0;
  const int vrem = KIND == kEpiNorm ? s.plain_nblocks - vbase * ng : 0;
  auto plain_count = [&](int g, int mq) { return vbase + ((g + mq) % ng < vrem ? 1 : 0); };
  auto unit_len = [&](int u) { return s.unit_tiles + plain_count(u % ng, u / ng); };
  if constexpr (KIND == kEpiNorm) {
    const int G = t_step, c = t_first;
    seq_units = s.units / G + (c < s.units - (s.units / G) * G ? 1 : 0);
    for (int j = 0; j < seq_units; ++j) my_count += unit_len(t_first + j * t_step);
  } else {
    my_count = t_first < s.tiles ? (s.tiles - 1 - t_first) / t_step + 1 : 0;
  }
  auto coords = [&](int i, int& m_blk, int& n_blk, int& upos) {
    if constexpr (KIND == kEpiNorm) {
      int u = t_first, len = unit_len(u);
      while (i >= len) {  // walk to the unit holding position i (a few units per CTA)
        i -= len;
        u += t_step;
        len = unit_len(u);
      }
      const int mq = u / ng;
      const int g = u - mq * ng;
      if (i < s.unit_tiles) {
        upos = i;
        n_blk = g * s.unit_tiles + i;
      } else {
        upos = -1;
        int v0 = 0;  // this group's first plain tile of the row group: the lower groups' shares
        for (int g2 = 0; g2 < g; ++g2) v0 += plain_count(g2, mq);
        n_blk = ng * s.unit_tiles + v0 + (i - s.unit_tiles);
      }
      m_blk = PAIR ? 2 * mq + cta_rank : mq;
    } else {
      tile_coords(t_first + i * t_step, m_blk, n_blk);
      upos = -1;
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], kTemptyCount);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&cload_bar[i], 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.has_out_map) tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();  // both CTAs' barriers initialized before any cross-CTA signal
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ----------------------------- TMA producer -----------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < my_count; ++i) {
        int m_blk, n_blk, upos;
        coords(i, m_blk, n_blk, upos);
        for (int kb = 0; kb < s.k_blocks; ++kb) {
          if (!wait_parity<PAIR>(&empty_bar[stage], phase ^ 1u, kSiteProducerEmpty)) goto producer_done;
          uint8_t* st = stage_base + stage * SB;
          if constexpr (PAIR) {
            // Both CTAs' loads complete on the leader's full barrier; only the leader arms it.
            const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if (cta_rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * SB);
            tma_load_2d_pair(st, &tmA, fb, kb * BK, m_blk * BM);
            tma_load_2d_pair(st + kTileABytes, &tmB, fb, kb * BK, n_blk * BN + cta_rank * (BN / 2));
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], SB);
            tma_load_2d(st, &tmA, &full_bar[stage], kb * BK, m_blk * BM);
            tma_load_2d(st + kTileABytes, &tmB, &full_bar[stage], kb * BK, n_blk * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: do not leave the CTA while TMA writes into its shared memory are pending.
      for (int i = 0; i < STAGES; ++i) {
        if (!wait_parity<PAIR>(&empty_bar[stage], phase ^ 1u, kSiteDrain)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    producer_done:;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------- MMA issuer -------------------------------
    // Pair: the leader (rank 0) issues cta_group::2 MMAs over both CTAs' stages and signals
    // both CTAs' barriers (one commit per barrier); the peer's warp 1 only owns TMEM.
    if (lane == 0 && cta_rank == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(PAIR ? 2 * BM : BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      for (int it = 0; it < my_count; ++it) {
        const int buf = it & 1;
        const uint32_t tphase = (it >> 1) & 1;
        if (!wait_parity<PAIR>(&tempty_bar[buf], tphase ^ 1u, kSiteMmaTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < s.k_blocks; ++kb) {
          if (!wait_parity<PAIR>(&full_bar[stage], phase, kSiteMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_base + stage * SB);
          const uint64_t a_desc = smem_desc_sw128(a_addr);
          const uint64_t b_desc = smem_desc_sw128(a_addr + kTileABytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // Advance 16 bf16 (32 bytes) along K inside the swizzle atom: +2 in addr>>4.
            if constexpr (PAIR) {
              mma_bf16_pair(d_tmem, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
            } else {
              mma_bf16(d_tmem, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
          if constexpr (PAIR) {
            mma_commit_pair(smem_u32(&empty_bar[stage]));
            mma_commit_pair(mapa_shared(smem_u32(&empty_bar[stage]), 1));
          } else {
            mma_commit(&empty_bar[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          mma_commit_pair(smem_u32(&tfull_bar[buf]));
          mma_commit_pair(mapa_shared(smem_u32(&tfull_bar[buf]), 1));
        } else {
          mma_commit(&tfull_bar[buf]);
        }
      }
    }
    __syncwarp();
  } else {
    // ----------------------------- Epilogue ---------------------------------
    // Warps 2..9. Warp w may access TMEM lanes [32*(w%4), 32*(w%4)+32), so its thread owns
    // accumulator row r = 32*(w%4) + lane. Warps 2..5 take the tile's columns [0, 128),
    // warps 6..9 columns [128, 256): two warps per scheduler hide each other's latency.
    // The residual epilogue (bandwidth-bound, shared-memory limited) uses warps 2..5 only.
    const int ew = warp - 2;          // 0..7
    const int wq = warp & 3;          // TMEM lane quadrant
    const int half = ew >> 2;         // column half of the tile
    const int ht = (ew & 3) * 32 + lane;  // thread index inside its half, 0..127
    const int r = wq * 32 + lane;     // accumulator row inside the tile
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const int col_base = half * (BN / 2);
    // Hand accumulator buffer b back to the MMA issuer (the pair leader's barrier in pair mode).
    auto release_acc = [&](int b) {
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[b]), 0));
      } else {
        mbar_arrive(&tempty_bar[b]);
      }
    };

    if constexpr (KIND == kEpiAct || KIND == kEpiNorm) {
      constexpr int kChunks = (BN / 2) / 32;  // 32-column chunks per half
      static_assert(kChunks % 2 == 0, "exchange stores pair up the chunks of a half");
      // Per-warp staging: two 32-row x 32-column bf16 buffers (64-byte swizzle) per warp, each
      // stored by the warp's own TMA store, so the warps of a half never wait on each other.
      uint8_t* stg_warp_ptr = epi_base + ew * 2 * kWarpStgBytes;
      const uint32_t stg_warp = smem_u32(stg_warp_ptr);
      const bool use_ln = p.ln.csum != nullptr;
      int sbuf = 0;
      // kEpiNorm: this thread's sum of squares of its row over the current unit's columns of
      // its half, and the two halves' sums exchanged at the end of each unit.
      uint64_t unit_ss2 = f2_pack(0.f, 0.f);
      float* ss_x = reinterpret_cast<float*>(epi_base + 8 * 2 * kWarpStgBytes);  // [2][BM]
      const uint64_t keep_policy = KIND == kEpiNorm ? l2_policy_evict_last() : 0ull;
      // kEpiNorm: the last finished unit whose normalize pass is pending; it runs in slices of
      // BM / unit_tiles rows, one after each following tile's epilogue, with the slice's rows
      // prefetched into L2 when that tile's iteration starts.
      int pend_mblk = -1, pend_g = 0, pend_slice = 0;
      for (int it = 0; it < my_count; ++it) {
        int m_blk, n_blk, upos;
        coords(it, m_blk, n_blk, upos);
        if constexpr (KIND == kEpiNorm) {
          if (pend_mblk >= 0)
            norm_prefetch_rows(p.norm, pend_mblk, pend_g, s.M, ew, lane, pend_slice * BM / s.unit_tiles,
                               (pend_slice + 1) * BM / s.unit_tiles);
        }
        const int warp_row0 = m_blk * BM + wq * 32;
        const bool rows_any = warp_row0 < s.M;  // this warp's 32 rows hold data
        const int buf = it & 1;
        const uint32_t tphase = (it >> 1) & 1;
        const int row = m_blk * BM + r;
        const bool row_ok = row < s.M;
        const int nh = n_blk * BN + col_base;  // first column of this half
        // What does not need the accumulator happens before waiting for it: the row's
        // LayerNorm statistics and an L1 prefetch of the half's per-column vectors.
        float mu = 0.f, rstd = 1.f;
        if (use_ln && row_ok) ln_row_stats(p.ln, row, mu, rstd);
        if (lane < 4 && nh + lane * 32 < s.N) {
          if (use_ln) prefetch_l1(p.ln.csum + nh + lane * 32);
          if (p.vec != nullptr) prefetch_l1(p.vec + nh + lane * 32);
        }
        const float nmr = -mu * rstd;
        {
          const bool ok = wait_parity<PAIR>(&tfull_bar[buf], tphase, kSiteEpiTmemFull);
          if (named_bar_any(3, 2 * kEpiThreads, !ok)) break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem_base + lane_off + buf * BN + col_base;
        // RMSNorm partials: this half's 128 columns form one partial block (kEpiAct), or
        // the running sum over the unit (kEpiNorm).
        const bool ss_on = KIND == kEpiNorm ? upos >= 0 : (p.ss_part != nullptr && nh < p.ss_cols);
        uint64_t ss2 = KIND == kEpiNorm ? unit_ss2 : f2_pack(0.f, 0.f);
#pragma unroll 1
        for (int c = 0; c < kChunks; ++c) {
          const int n0 = nh + c * 32;
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          if (c == kChunks - 1) release_acc(buf);
          if (n0 >= s.N) continue;  // uniform inside the half
          // acc -> rstd * (acc - mu * csum) + vec  (= fma(acc, rstd, fma(-mu rstd, csum, vec))),
          // two columns per packed instruction
          if (use_ln) {
            const float4* cp = reinterpret_cast<const float4*>(p.ln.csum + n0);
            const float4* bp = reinterpret_cast<const float4*>(p.vec + n0);
            const uint64_t rs2 = f2_pack(rstd, rstd);
            const uint64_t nm2 = f2_pack(nmr, nmr);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 c4 = __ldg(cp + q);
              float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
              if (p.vec != nullptr) b4 = __ldg(bp + q);
              const uint64_t t0 = ffma2(nm2, f2_pack(c4.x, c4.y), f2_pack(b4.x, b4.y));
              const uint64_t t1 = ffma2(nm2, f2_pack(c4.z, c4.w), f2_pack(b4.z, b4.w));
              f2_unpack(ffma2(f2_pack(v[4 * q], v[4 * q + 1]), rs2, t0), v[4 * q], v[4 * q + 1]);
              f2_unpack(ffma2(f2_pack(v[4 * q + 2], v[4 * q + 3]), rs2, t1), v[4 * q + 2], v[4 * q + 3]);
            }
          } else if (p.vec != nullptr) {
            const float4* bp = reinterpret_cast<const float4*>(p.vec + n0);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 b4 = __ldg(bp + q);
              v[4 * q] += b4.x;
              v[4 * q + 1] += b4.y;
              v[4 * q + 2] += b4.z;
              v[4 * q + 3] += b4.w;
            }
          }
          if (p.act == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j) gelu_tanh2(v[2 * j], v[2 * j + 1]);
          }
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
          if (ss_on) {
            // WanRMSNorm normalizes the bf16 Linear output: square the rounded values.
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float2 f = unpack_bf16x2(w[j]);
              const uint64_t f2 = f2_pack(f.x, f.y);
              ss2 = ffma2(f2, f2, ss2);
            }
          }
          if (KIND == kEpiNorm && upos < 0 && p.xchg.P > 0) {
            // Token-sharded run: a plain (v) tile goes into the exchange region of the rank
            // owning its unit. Two consecutive chunks fill the warp's two staging buffers as one
            // 32-row x 128-byte block (16-byte pieces XOR-swizzled by row); the block then
            // leaves as whole 128-byte lines, 4 rows per store instruction (a head's token row
            // is 256 contiguous bytes at the destination, so each line is one NVLink write).
            const int pbase = (c & 1) * 4;
            if (pbase == 0) {
              if (lane == 0) bulk_wait_read<0>();  // earlier TMA stores have read the buffers
              __syncwarp();
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st_shared_v4(stg_warp + lane * 128 + (((pbase + q) ^ (lane & 7)) << 4), w[4 * q], w[4 * q + 1],
                           w[4 * q + 2], w[4 * q + 3]);
            if (pbase != 0) {
              __syncwarp();
              const XchgParams& xc = p.xchg;
              const int vcol = n0 - 32 - s.norm_groups * p.norm.width;  // first column of the pair
              const int pc = lane & 7;
#pragma unroll 2
              for (int i = 0; i < 8; ++i) {
                const int rr = 4 * i + (lane >> 3);
                const uint4 val = ld_shared_u4(stg_warp + rr * 128 + ((pc ^ (rr & 7)) << 4));
                const int grow = warp_row0 + rr;
                if (grow < s.M) {
                  const int b = grow / xc.Lp;
                  const int gtok = xc.rank * xc.Lp + (grow - b * xc.Lp);
                  st_global_v4(xchg_addr(xc, 2, b, gtok, vcol) + pc * 16, val.x, val.y, val.z, val.w);
                }
              }
              __syncwarp();  // the block is read out before the next chunk is staged
            }
            continue;
          }
          // Stage the warp's 32 rows x 32 bf16 (64-byte swizzle) and store them with TMA.
          if (lane == 0) bulk_wait_read<1>();  // the store that last used this buffer has read it
          __syncwarp();
          const uint32_t rowa = stg_warp + sbuf * kWarpStgBytes + lane * 64;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            st_shared_v4(rowa + ((q ^ ((lane >> 1) & 3)) << 4), w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (rows_any) {
              if (KIND == kEpiNorm && ss_on) {  // read back by this CTA's normalize pass soon
                tma_store_2d_hint(&tmOut, stg_warp_ptr + sbuf * kWarpStgBytes, n0, warp_row0, keep_policy);
              } else {
                tma_store_2d(&tmOut, stg_warp_ptr + sbuf * kWarpStgBytes, n0, warp_row0);
              }
            }
            bulk_commit();
          }
          sbuf ^= 1;
        }
        if constexpr (KIND == kEpiNorm) {
          unit_ss2 = ss2;
          if (pend_mblk >= 0) {
            norm_pass_rows(p.norm, p.xchg, ss_x, pend_mblk, pend_g, s.M, p.rows_per_batch, ew, lane,
                           pend_slice * BM / s.unit_tiles, (pend_slice + 1) * BM / s.unit_tiles);
            if (++pend_slice == s.unit_tiles) pend_mblk = -1;
          }
          if (upos == s.unit_tiles - 1) {
            // Unit done. The previous unit's last slice ran just above in every warp: wait for
            // all of them before its sums of squares are overwritten. Then publish this unit's
            // halves' sums and make this CTA's TMA stores of the unit visible to generic loads.
            named_bar_sync(5, 2 * kEpiThreads);
            float s0, s1;
            f2_unpack(unit_ss2, s0, s1);
            ss_x[half * BM + r] = s0 + s1;
            unit_ss2 = f2_pack(0.f, 0.f);
            if (lane == 0) {
              bulk_wait_all<0>();
              fence_proxy_async_global();
            }
            __syncwarp();
            named_bar_sync(5, 2 * kEpiThreads);
            pend_mblk = m_blk;
            pend_g = n_blk / s.unit_tiles;
            pend_slice = 0;
          }
        } else {
          if (ss_on && row_ok) {
            float s0, s1;
            f2_unpack(ss2, s0, s1);
            p.ss_part[static_cast<size_t>(row) * p.ss_ld + (nh >> 7)] = (s0 + s1) * (1.f / 128.f);
          }
        }
      }
      if constexpr (KIND == kEpiNorm) {
        // the last unit's remaining rows (no tile left to hide them behind)
        if (pend_mblk >= 0)
          norm_pass_rows(p.norm, p.xchg, ss_x, pend_mblk, pend_g, s.M, p.rows_per_batch, ew, lane,
                         pend_slice * BM / s.unit_tiles, BM);
      }
      if (lane == 0) bulk_wait_all<0>();
    } else if (half < Cfg<KIND>::kHalves) {
      // ----------------------------- residual -----------------------------
      // kHalves = 1: warps 2-5 process the tile's eight 32-column chunks in turn.
      // kHalves = 2: half h (warps 2-5 / 6-9) processes chunks h, h + 2, h + 4, h + 6; each half
      // owns every other residual buffer and one bf16 staging buffer, issues its own loads and
      // stores, and the halves merge their row statistics through shared memory per tile.
      constexpr int HV = Cfg<KIND>::kHalves;
      const int et = ht;          // thread index inside the half
      const bool lead = et == 0;  // issues this half's TMA loads and stores
      constexpr int NB = Cfg<KIND>::kNumCBuf;  // residual buffers in all
      constexpr int NBH = NB / HV;             // ... per half
      constexpr int LA = Cfg<KIND>::kLookahead;  // chunks requested ahead, per half
      static_assert(LA >= 1 && LA < NBH, "lookahead must leave one buffer being stored");
      constexpr int CPT = BN / 32;  // 32-column chunks per tile
      constexpr int CPH = CPT / HV;  // ... per half
      constexpr bool XS = Cfg<KIND>::kXStaged;
      static_assert(HV == 1 || !XS || NBH - LA - 1 == 0, "one staging buffer per half needs drained stores");
      uint8_t* cbuf0 = epi_base;
      uint8_t* xbuf0 = epi_base + NB * 16384;
      float* st_x = reinterpret_cast<float*>(epi_base + NB * 16384 + (XS ? 2 * kStgBytes : 0u));  // [128][3]
      const int my_tiles = (t_first < s.tiles) ? (s.tiles - 1 - t_first) / t_step + 1 : 0;
      const int total_k = my_tiles * CPH;
      const bool has_x = p.has_x_map;
      auto buf_of = [&](int k) { return half + HV * (k % NBH); };
      // This half's k-th chunk -> (tile, column chunk); issue its residual load.
      auto issue_load = [&](int k) {
        const int ti = k / CPH;
        const int c = half + HV * (k - ti * CPH);
        int m_blk, n_blk;
        tile_coords(t_first + ti * t_step, m_blk, n_blk);
        const int n0 = n_blk * BN + c * 32;
        const int bi = buf_of(k);
        uint64_t* bar = &cload_bar[bi];
        mbar_arrive_expect_tx(bar, 16384);
        tma_load_2d(cbuf0 + bi * 16384, &tmC, bar, n0 < s.N ? n0 : 0, m_blk * BM);
      };
      if (lead) {
        for (int k = 0; k < LA && k < total_k; ++k) issue_load(k);
      }
      int k = 0;
      bool failed = false;
      for (int ti = 0; ti < my_tiles; ++ti) {
        int m_blk, n_blk;
        tile_coords(t_first + ti * t_step, m_blk, n_blk);
        const bool rows_any = m_blk * BM < s.M;  // false only for a pair's trailing half
        const int buf = ti & 1;
        const uint32_t tphase = (ti >> 1) & 1;
        {
          const bool ok = wait_parity<PAIR>(&tfull_bar[buf], tphase, kSiteEpiTmemFull);
          if (named_bar_any(3, HV * kEpiThreads, !ok)) {
            failed = true;
            break;
          }
        }
        tc_fence_after();
        const int row = m_blk * BM + r;
        const int batch = (row < s.M ? row : s.M - 1) / p.rows_per_batch;
        const float* gb = p.gate_b != nullptr ? p.gate_b + static_cast<size_t>(batch) * p.gate_b_stride : nullptr;
        float run_n = 0.f, run_mean = 0.f, run_m2 = 0.f;
#pragma unroll 1
        for (int j = 0; j < CPH; ++j, ++k) {
          const int c = half + HV * j;
          const int n0 = n_blk * BN + c * 32;
          const int bi = buf_of(k);
          const int xs = HV == 1 ? (k & 1) : half;  // bf16 staging buffer of this chunk
          if (lead) {
            // The buffer of chunk k + LA last held chunk k + LA - NBH: its store must have been read.
            bulk_wait_read<NBH - LA - 1>();
            if (k + LA < total_k) issue_load(k + LA);
          }
          named_bar_sync(1 + half, kEpiThreads);
          float acc[32];
          tmem_ld32(tmem_base + lane_off + buf * BN + c * 32, acc);
          if (j == CPH - 1) {
            release_acc(buf);
          }
          const bool c_ok = wait_parity(&cload_bar[bi], (k / NBH) & 1, kSiteEpiCLoad);
          const bool col_ok = n0 < s.N;
          const uint32_t crow = smem_u32(cbuf0 + bi * 16384) + r * 128;
          float out[32];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            ld_shared_v4(crow + ((q ^ (r & 7)) << 4), out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
          }
          if (col_ok) {
            const float4* bp = reinterpret_cast<const float4*>(p.vec + n0);
            const float4* gp = p.gate_a != nullptr ? reinterpret_cast<const float4*>(p.gate_a + n0) : nullptr;
            const float4* gbp = gb != nullptr ? reinterpret_cast<const float4*>(gb + n0) : nullptr;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float bb[4] = {0.f, 0.f, 0.f, 0.f};
              if (p.vec != nullptr) {
                const float4 t = __ldg(bp + q);
                bb[0] = t.x; bb[1] = t.y; bb[2] = t.z; bb[3] = t.w;
              }
              if (gp != nullptr) {
                const float4 t = __ldg(gp + q);
                float gg[4] = {t.x, t.y, t.z, t.w};
                if (gbp != nullptr) {
                  const float4 u = __ldg(gbp + q);
                  gg[0] += u.x; gg[1] += u.y; gg[2] += u.z; gg[3] += u.w;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) out[4 * q + i] = fmaf(acc[4 * q + i] + bb[i], gg[i], out[4 * q + i]);
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) out[4 * q + i] += acc[4 * q + i] + bb[i];
              }
            }
          }
          // Write the result back in place (same swizzled slots) for the TMA store.
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            st_shared_v4(crow + ((q ^ (r & 7)) << 4), __float_as_uint(out[4 * q]), __float_as_uint(out[4 * q + 1]),
                         __float_as_uint(out[4 * q + 2]), __float_as_uint(out[4 * q + 3]));
          }
          if (col_ok && p.stats_out != nullptr) {
            // Chunk (mean, M2), merged into the running per-row statistics (Chan). Four
            // independent accumulators keep the dependency chains short.
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 32; ++i) s4[i & 3] += out[i];
            const float cmean = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.f / 32.f);
            float m4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float d = out[i] - cmean;
              m4[i & 3] = fmaf(d, d, m4[i & 3]);
            }
            const float cm2 = (m4[0] + m4[1]) + (m4[2] + m4[3]);
            const float tot = run_n + 32.f;
            const float delta = cmean - run_mean;
            run_mean += delta * (32.f / tot);
            run_m2 += cm2 + delta * delta * (run_n * 32.f / tot);
            run_n = tot;
          }
          if (XS && has_x) {
            const uint32_t xrow = smem_u32(xbuf0 + xs * kStgBytes) + r * 64;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              st_shared_v4(xrow + ((q ^ ((r >> 1) & 3)) << 4), pack_bf16x2(out[8 * q], out[8 * q + 1]),
                           pack_bf16x2(out[8 * q + 2], out[8 * q + 3]), pack_bf16x2(out[8 * q + 4], out[8 * q + 5]),
                           pack_bf16x2(out[8 * q + 6], out[8 * q + 7]));
            }
          }
          if (!XS && has_x && col_ok && row < s.M) {
            // bf16 copy of the updated row chunk, stored straight from registers (64 bytes).
            uint8_t* dst = reinterpret_cast<uint8_t*>(p.x_out) + (static_cast<size_t>(row) * p.ldx + n0) * 2;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              st_global_v4(dst + 16 * q, pack_bf16x2(out[8 * q], out[8 * q + 1]), pack_bf16x2(out[8 * q + 2], out[8 * q + 3]),
                           pack_bf16x2(out[8 * q + 4], out[8 * q + 5]), pack_bf16x2(out[8 * q + 6], out[8 * q + 7]));
            }
          }
          fence_proxy_async_smem();
          // A residual load that did not arrive fails the chunk; the halves decide together at
          // the end of the tile (no early exit here, so both halves keep meeting the same barriers).
          if (named_bar_any(1 + half, kEpiThreads, !c_ok)) failed = true;
          if (lead) {
            if (col_ok && rows_any && !failed) {
              tma_store_2d(&tmOut, cbuf0 + bi * 16384, n0, m_blk * BM);
              if (XS && has_x) tma_store_2d(&tmX, xbuf0 + xs * kStgBytes, n0, m_blk * BM);
            }
            bulk_commit();
          }
        }
        if (HV == 2 && half == 1 && p.stats_out != nullptr) {
          st_x[3 * r] = run_n;
          st_x[3 * r + 1] = run_mean;
          st_x[3 * r + 2] = run_m2;
        }
        if (named_bar_any(3, HV * kEpiThreads, failed)) {
          failed = true;
          break;
        }
        if (half == 0 && p.stats_out != nullptr && row < s.M) {
          if (HV == 2) {
            // Chan merge with the other half's statistics of the same row.
            const float n1 = st_x[3 * r];
            if (n1 > 0.f) {
              const float tot = run_n + n1;
              const float delta = st_x[3 * r + 1] - run_mean;
              run_mean += delta * (n1 / tot);
              run_m2 += st_x[3 * r + 2] + delta * delta * (run_n * n1 / tot);
              run_n = tot;
            }
          }
          const int ntiles = (s.N + BN - 1) / BN;
          *reinterpret_cast<float2*>(p.stats_out + (static_cast<size_t>(row) * ntiles + n_blk) * 2) =
              make_float2(run_mean, run_m2);
        }
      }
      if (lead) bulk_wait_all<0>();
      // Do not leave with residual loads in flight (only reachable after a failure).
      if (failed && lead) {
        for (int kk = k; kk < k + LA && kk < total_k; ++kk) {
          wait_parity(&cload_bar[buf_of(kk)], (kk / NBH) & 1, kSiteDrain);
        }
      }
    }
  }

  if constexpr (KIND == kEpiNorm) {
    if (p.xchg.P > 0) __threadfence_system();  // this thread's stores into peer regions are visible
  }
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();  // neither CTA leaves while the other may still signal or read it
  } else {
    __syncthreads();
  }
  if constexpr (KIND == kEpiNorm) {
    // The last CTA to finish publishes the exchange epoch into flags[rank] of every region
    // (system-scope release), after which the owners may read what this rank stored.
    if (p.xchg.P > 0 && threadIdx.x == 0) {
      const XchgParams& xc = p.xchg;
      if (atomicAdd(xc.done_ctr, 1u) == gridDim.x - 1) {
        __threadfence_system();
        for (int q = 0; q < xc.P; ++q) {
          unsigned int* f = reinterpret_cast<unsigned int*>(xc.base[q] + xc.flag_off) + xc.rank;
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(xc.epoch) : "memory");
        }
        atomicExch(xc.done_ctr, 0u);
      }
    }
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem_base, kTmemCols);
    } else {
      tmem_dealloc(tmem_base, kTmemCols);
    }
  }
}

// Self-test of the bounded-wait path: one thread waits for `flag` to become nonzero with the
// library's wait limit; when nothing sets it the wait gives up, records kErrTimeout /
// kSiteSelfTest in the error record and the kernel returns normally.
__global__ void wait_selftest_kernel(const unsigned int* flag) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = g_wdit_wait_limit_ns;
  while (ld_acquire_gpu(flag) == 0u) {
    if (globaltimer_ns() - t0 > limit) {
      report_error(kErrTimeout, kSiteSelfTest, 0u);
      return;
    }
    __nanosleep(1000);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool get_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return g_encode != nullptr;
}

int make_map(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* ptr, int inner, int outer,
             long long row_stride_elems, int box_inner, int box_outer, CUtensorMapSwizzle sw) {
  if (!get_encoder()) return WDIT_ERR_DRIVER;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return WDIT_ERR_ALIGN;
  if (((row_stride_elems * esize) & 15) != 0) return WDIT_ERR_ALIGN;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems * esize)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? WDIT_OK : WDIT_ERR_TMAP;
}

int g_num_sms = 0;

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_num_sms;
}

// Whether the tensor-bound variants (bias/GELU, long-K residual) run on CTA pairs.
int g_cta_pair = 1;
unsigned long long g_wait_limit_host = 2000000000ull;  // host copy of g_wdit_wait_limit_ns
std::mutex g_err_ptr_mutex;
unsigned int* g_err_ptr[64] = {};

template <int KIND, bool PAIR>
int launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o, const CUtensorMap& c,
           const CUtensorMap& x, const GemmShape& shape, const EpiParams& p, cudaStream_t stream, int max_ctas) {
  static bool attr_set[64] = {};
  static int pair_slots[64] = {};  // co-resident CTA pairs per device
  int dev = 0;
  cudaGetDevice(&dev);
  constexpr uint32_t smem = smem_bytes<KIND, PAIR>();
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(num_threads<KIND>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 1 : 0;
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<KIND, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
    if (PAIR) {
      int n = 0;
      cfg.gridDim = dim3(2);
      e = cudaOccupancyMaxActiveClusters(&n, gemm_kernel<KIND, PAIR>, &cfg);
      if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
      if (n <= 0) return WDIT_ERR_CUDA_BASE + static_cast<int>(cudaErrorInvalidConfiguration);
      pair_slots[dev & 63] = n;
    }
    attr_set[dev & 63] = true;
  }
  GemmShape s = shape;
  int grid = num_sms();
  if (s.norm_groups > 0) s.units = (PAIR ? (s.m_blocks + 1) / 2 : s.m_blocks) * s.norm_groups;
  if (PAIR) {
    s.tiles = ((s.m_blocks + 1) / 2) * s.n_blocks;  // 256-row pair tiles
    grid = 2 * pair_slots[dev & 63];
    if (max_ctas > 0 && max_ctas < grid) grid = max_ctas < 2 ? 2 : max_ctas & ~1;
    if (2 * s.tiles < grid) grid = 2 * s.tiles;
  } else {
    if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
    if (s.tiles < grid) grid = s.tiles;
  }
  if (grid <= 0) return WDIT_OK;
  cfg.gridDim = dim3(grid);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_kernel<KIND, PAIR>, a, b, o, c, x, s, p);
  return e == cudaSuccess ? WDIT_OK : WDIT_ERR_CUDA_BASE + static_cast<int>(e);
}

int check_common(const void* A, int lda, const void* B, int ldb, int M, int N, int K) {
  if (A == nullptr || B == nullptr) return WDIT_ERR_ARG;
  if (M <= 0 || N <= 0 || K <= 0) return WDIT_ERR_SHAPE;
  if (N % 64 != 0 || K % 8 != 0) return WDIT_ERR_SHAPE;
  if (lda < K || ldb < K) return WDIT_ERR_SHAPE;
  return WDIT_OK;
}

GemmShape make_shape(int M, int N, int K) {
  GemmShape s = {};
  s.M = M;
  s.N = N;
  s.K = K;
  s.raster_rows = static_cast<long long>(N) * K * 2 > kRasterBBytes ? kRasterRows : 1;
  s.m_blocks = (M + BM - 1) / BM;
  s.n_blocks = (N + BN - 1) / BN;
  s.k_blocks = (K + BK - 1) / BK;
  s.tiles = s.m_blocks * s.n_blocks;
  return s;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// pair: each CTA of a pair loads one 128-row half of the B tile.
int build_ab(CUtensorMap* ma, CUtensorMap* mb, const void* A, int lda, const void* B, int ldb, int M, int N, int K,
             bool pair = false) {
  int rc = make_map(ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, K, M, lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return make_map(mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, K, N, ldb, BK, pair ? BN / 2 : BN,
                  CU_TENSOR_MAP_SWIZZLE_128B);
}

// Pairs pay off once there are several 256-row blocks to spread over the GPU.
bool use_pair(int M) { return g_cta_pair != 0 && M > 2 * BM; }

int ln_fill(LnFold* ln, const float* csum, const float* stats, int stats_tiles, int stats_width, int row_len,
            float eps) {
  ln->csum = csum;
  ln->stats = stats;
  ln->stats_tiles = stats_tiles;
  ln->stats_width = stats_width;
  ln->row_len = row_len;
  ln->eps = eps;
  if (csum != nullptr) {
    if (stats == nullptr || stats_tiles <= 0 || stats_width <= 0 || row_len <= 0) return WDIT_ERR_ARG;
    if (!aligned16(csum) || (reinterpret_cast<uintptr_t>(stats) & 7) != 0) return WDIT_ERR_ALIGN;
  }
  return WDIT_OK;
}

// RMSNorm partials: one fp32 mean square per row and 128-column block of the normalized
// groups, rows of norm_groups * norm_width / 128 entries (256-byte rounded).
long long norm_partials_bytes(int M, int norm_groups, int norm_width) {
  const long long cols = static_cast<long long>(norm_groups) * (norm_width / 128);
  return ((static_cast<long long>(M) * cols * 4 + 255) / 256) * 256;
}

int check_norm(const void* A, int lda, const void* B, int ldb, const void* out, int ldo, int M, int N, int K,
               const float* vec, int norm_groups, int norm_width, const float* norm_w0, const float* norm_w1,
               int rope_groups, const float* rope_cos, const float* rope_sin, int rope_ld, int rows_per_batch,
               int token_offset) {
  int rc = check_common(A, lda, B, ldb, M, N, K);
  if (rc) return rc;
  if (out == nullptr || ldo < N) return WDIT_ERR_ARG;
  if (!aligned16(out) || ldo % 8 != 0) return WDIT_ERR_ALIGN;
  if (norm_groups < 0 || norm_groups > 2 || rope_groups < 0 || rope_groups > norm_groups) return WDIT_ERR_ARG;
  if (norm_groups > 0) {
    if (norm_width <= 0 || norm_width % 128 != 0 || norm_groups * norm_width > N) return WDIT_ERR_SHAPE;
    if (norm_w0 == nullptr || (norm_groups > 1 && norm_w1 == nullptr)) return WDIT_ERR_ARG;
    if (!aligned16(norm_w0) || (norm_w1 && !aligned16(norm_w1))) return WDIT_ERR_ALIGN;
  }
  if (rope_groups > 0) {
    // token-major tables: entry (token, pair) at token * rope_ld + pair, 64 pairs per head
    if (rope_cos == nullptr || rope_sin == nullptr || rows_per_batch <= 0 || token_offset < 0) return WDIT_ERR_ARG;
    if (rope_ld < 64) return WDIT_ERR_SHAPE;
    if (!aligned16(rope_cos) || !aligned16(rope_sin) || rope_ld % 4 != 0) return WDIT_ERR_ALIGN;
  }
  if (vec != nullptr && !aligned16(vec)) return WDIT_ERR_ALIGN;
  return WDIT_OK;
}

// GEMM (bias / absorbed LayerNorm, bf16 out, RMSNorm partials) followed by the in-place
// RMSNorm / RoPE pass over the normalized column groups.
int run_norm(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
             const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles, int ln_stats_width,
             float ln_eps, int norm_groups, int norm_width, const float* norm_w0, const float* norm_w1,
             float norm_eps, int rope_groups, const float* rope_cos, const float* rope_sin, int rope_ld,
             int rows_per_batch, int token_offset, float* part, cudaStream_t stream, int max_ctas) {
  EpiParams p = {};
  int rc = ln_fill(&p.ln, ln_csum, ln_stats, ln_stats_tiles, ln_stats_width, K, ln_eps);
  if (rc) return rc;
  p.vec = vec;
  p.rows_per_batch = M;
  p.has_out_map = 1;
  if (norm_groups > 0) {
    p.ss_part = part;
    p.ss_ld = norm_groups * (norm_width / 128);
    p.ss_cols = norm_groups * norm_width;
  }
  const bool pair = use_pair(M);
  CUtensorMap ma, mb, mo, none;
  memset(&none, 0, sizeof(none));
  if ((rc = build_ab(&ma, &mb, A, lda, B, ldb, M, N, K, pair))) return rc;
  if ((rc = make_map(&mo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, N, M, ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  const GemmShape shape = make_shape(M, N, K);
  rc = pair ? launch<kEpiAct, true>(ma, mb, mo, none, none, shape, p, stream, max_ctas)
            : launch<kEpiAct, false>(ma, mb, mo, none, none, shape, p, stream, max_ctas);
  if (rc || norm_groups == 0) return rc;
  return launch_rms_rope_apply(out, ldo, M, part, p.ss_ld, norm_groups, norm_width, norm_w0, norm_w1, norm_eps,
                               rope_groups, rope_cos, rope_sin, rope_ld, rows_per_batch > 0 ? rows_per_batch : M,
                               token_offset, stream);
}

// The same result in one launch: the norm GEMM with the RMSNorm / RoPE in its epilogue.
int run_norm_fused(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                   const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                   int ln_stats_width, float ln_eps, int norm_groups, int norm_width, const float* norm_w0,
                   const float* norm_w1, float norm_eps, int rope_groups, const float* rope_cos,
                   const float* rope_sin, int rope_ld, int rows_per_batch, int token_offset, cudaStream_t stream,
                   int max_ctas, const XchgParams* xchg = nullptr) {
  EpiParams p = {};
  if (xchg != nullptr) p.xchg = *xchg;
  int rc = ln_fill(&p.ln, ln_csum, ln_stats, ln_stats_tiles, ln_stats_width, K, ln_eps);
  if (rc) return rc;
  p.vec = vec;
  p.rows_per_batch = rows_per_batch > 0 ? rows_per_batch : M;
  p.has_out_map = 1;
  NormParams& np = p.norm;
  np.out = out;
  np.ldo = ldo;
  np.width = norm_width;
  np.inv_width = 1.f / static_cast<float>(norm_width);
  np.eps = norm_eps;
  np.w0 = norm_w0;
  np.w1 = norm_w1;
  np.rope_groups = rope_groups;
  np.cos = rope_cos;
  np.sin = rope_sin;
  np.rope_ld = rope_ld;
  np.token_offset = token_offset;
  const bool pair = use_pair(M);
  CUtensorMap ma, mb, mo, none;
  memset(&none, 0, sizeof(none));
  if ((rc = build_ab(&ma, &mb, A, lda, B, ldb, M, N, K, pair))) return rc;
  if ((rc = make_map(&mo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, N, M, ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  GemmShape shape = make_shape(M, N, K);
  shape.norm_groups = norm_groups;
  shape.unit_tiles = norm_width / BN;
  shape.plain_nblocks = shape.n_blocks - norm_groups * shape.unit_tiles;
  return pair ? launch<kEpiNorm, true>(ma, mb, mo, none, none, shape, p, stream, max_ctas)
              : launch<kEpiNorm, false>(ma, mb, mo, none, none, shape, p, stream, max_ctas);
}

}  // namespace

int error_record_ptr(unsigned int** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
  if (dev < 0 || dev >= 64) return WDIT_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_err_ptr_mutex);
  if (g_err_ptr[dev] == nullptr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_wdit_error);
    if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
    g_err_ptr[dev] = static_cast<unsigned int*>(addr);
  }
  *out = g_err_ptr[dev];
  return WDIT_OK;
}

unsigned long long wait_limit_ns() { return g_wait_limit_host; }

}  // namespace wdit

using namespace wdit;

extern "C" {

int wdit_stats_tile_width(void) { return BN; }

int wdit_num_sms(void) { return num_sms(); }

int wdit_set_cta_pair(int enable) {
  const int prev = g_cta_pair;
  g_cta_pair = enable != 0 ? 1 : 0;
  return prev;
}

int wdit_set_wait_limit_ns(unsigned long long ns) {
  cudaError_t e = cudaMemcpyToSymbol(g_wdit_wait_limit_ns, &ns, sizeof(ns));
  if (e == cudaSuccess) g_wait_limit_host = ns;
  return e == cudaSuccess ? WDIT_OK : WDIT_ERR_CUDA_BASE + static_cast<int>(e);
}

int wdit_wait_selftest(const unsigned int* flag, void* stream) {
  if (flag == nullptr) return WDIT_ERR_ARG;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WDIT_OK : WDIT_ERR_CUDA_BASE + static_cast<int>(e);
}

int wdit_read_error(unsigned int* out4, int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
  e = cudaMemcpyFromSymbol(out4, g_wdit_error, 4 * sizeof(unsigned int));
  if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
  if (clear) {
    unsigned int z[4] = {0, 0, 0, 0};
    e = cudaMemcpyToSymbol(g_wdit_error, z, sizeof(z));
    if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
  }
  return WDIT_OK;
}

int wdit_gemm_act(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                  const float* vec, int act, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                  int ln_stats_width, float ln_eps, float* ms_out, int ms_ld, int ms_cols, void* stream,
                  int max_ctas) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  int rc = check_common(A, lda, B, ldb, M, N, K);
  if (rc) return rc;
  if (out == nullptr || ldo < N) return WDIT_ERR_ARG;
  if (act != 0 && act != 1) return WDIT_ERR_ARG;
  if (vec != nullptr && !aligned16(vec)) return WDIT_ERR_ALIGN;
  if (ms_out != nullptr && (ms_cols <= 0 || ms_cols % 128 != 0 || ms_cols > N || ms_ld < ms_cols / 128))
    return WDIT_ERR_SHAPE;
  EpiParams p = {};
  rc = ln_fill(&p.ln, ln_csum, ln_stats, ln_stats_tiles, ln_stats_width, K, ln_eps);
  if (rc) return rc;
  p.vec = vec;
  p.act = act;
  p.rows_per_batch = M;
  p.has_out_map = 1;
  p.ss_part = ms_out;
  p.ss_ld = ms_ld;
  p.ss_cols = ms_out != nullptr ? ms_cols : 0;
  CUtensorMap ma, mb, mo, none;
  memset(&none, 0, sizeof(none));
  const bool pair = use_pair(M);
  if ((rc = build_ab(&ma, &mb, A, lda, B, ldb, M, N, K, pair))) return rc;
  if ((rc = make_map(&mo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, N, M, ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  if (pair)
    return launch<kEpiAct, true>(ma, mb, mo, none, none, make_shape(M, N, K), p, static_cast<cudaStream_t>(stream),
                                 max_ctas);
  return launch<kEpiAct, false>(ma, mb, mo, none, none, make_shape(M, N, K), p, static_cast<cudaStream_t>(stream),
                                max_ctas);
}

int wdit_gemm_residual(const void* A, int lda, const void* B, int ldb, const float* C, int ldc, float* out, int ldo,
                       int M, int N, int K, const float* bias, const float* gate_a, const float* gate_b,
                       int gate_b_stride, int rows_per_batch, void* x_bf16_out, int ldx, float* stats_out,
                       void* stream, int max_ctas) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  int rc = check_common(A, lda, B, ldb, M, N, K);
  if (rc) return rc;
  if (C == nullptr || out == nullptr || ldc < N || ldo < N) return WDIT_ERR_ARG;
  if (gate_b != nullptr && (gate_a == nullptr || rows_per_batch <= 0 || gate_b_stride < N)) return WDIT_ERR_ARG;
  if ((bias && !aligned16(bias)) || (gate_a && !aligned16(gate_a)) || (gate_b && !aligned16(gate_b)))
    return WDIT_ERR_ALIGN;
  if (gate_b != nullptr && (gate_b_stride % 4) != 0) return WDIT_ERR_ALIGN;
  if (x_bf16_out != nullptr && ldx < N) return WDIT_ERR_ARG;
  if (stats_out != nullptr && (reinterpret_cast<uintptr_t>(stats_out) & 7) != 0) return WDIT_ERR_ALIGN;
  // An in-place update must be exactly in place: every tile reads its residual before storing.
  if (C != out) {
    const char* c0 = reinterpret_cast<const char*>(C);
    const char* c1 = c0 + (static_cast<size_t>(M - 1) * ldc + N) * 4;
    const char* o0 = reinterpret_cast<const char*>(out);
    const char* o1 = o0 + (static_cast<size_t>(M - 1) * ldo + N) * 4;
    if (c0 < o1 && o0 < c1) return WDIT_ERR_ALIAS;
  } else if (ldc != ldo) {
    return WDIT_ERR_ALIAS;
  }
  EpiParams p = {};
  p.vec = bias;
  p.gate_a = gate_a;
  p.gate_b = gate_b;
  p.gate_b_stride = gate_b_stride;
  p.rows_per_batch = rows_per_batch > 0 ? rows_per_batch : M;
  p.stats_out = stats_out;
  p.has_out_map = 1;
  p.has_x_map = x_bf16_out != nullptr ? 1 : 0;
  p.x_out = x_bf16_out;
  p.ldx = ldx;
  CUtensorMap ma, mb, mo, mc, mx;
  memset(&mx, 0, sizeof(mx));
  // Long reductions are tensor-bound (deeper mainloop, CTA pairs), short ones HBM-bound
  // (deeper residual ring).
  const bool long_k = K >= 4096;
  const bool pair = long_k && use_pair(M);
  if ((rc = build_ab(&ma, &mb, A, lda, B, ldb, M, N, K, pair))) return rc;
  if ((rc = make_map(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out, N, M, ldo, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, C, N, M, ldc, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if (x_bf16_out != nullptr && (reinterpret_cast<uintptr_t>(x_bf16_out) & 15) != 0) return WDIT_ERR_ALIGN;
  if (x_bf16_out != nullptr && (ldx % 8) != 0) return WDIT_ERR_ALIGN;
  if (x_bf16_out != nullptr &&
      (rc = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x_bf16_out, N, M, ldx, 32, BM, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  const GemmShape shape = make_shape(M, N, K);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pair) return launch<kEpiResidualLongK, true>(ma, mb, mo, mc, mx, shape, p, st, max_ctas);
  if (long_k) return launch<kEpiResidualLongK, false>(ma, mb, mo, mc, mx, shape, p, st, max_ctas);
  return launch<kEpiResidual, false>(ma, mb, mo, mc, mx, shape, p, st, max_ctas);
}

long long wdit_gemm_norm_workspace_bytes(int M, int N, int norm_groups, int norm_width) {
  if (M <= 0 || norm_groups <= 0 || norm_width <= 0) return 0;
  (void)N;
  return norm_partials_bytes(M, norm_groups, norm_width);
}

int wdit_gemm_norm(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                   const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                   int ln_stats_width, float ln_eps, int norm_groups, int norm_width, const float* norm_w0,
                   const float* norm_w1, float norm_eps, int rope_groups, const float* rope_cos, const float* rope_sin,
                   int rope_ld, int rows_per_batch, int token_offset, void* workspace, long long workspace_bytes,
                   void* stream, int max_ctas) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  int rc = check_norm(A, lda, B, ldb, out, ldo, M, N, K, vec, norm_groups, norm_width, norm_w0, norm_w1, rope_groups,
                      rope_cos, rope_sin, rope_ld, rows_per_batch, token_offset);
  if (rc) return rc;
  if (norm_groups > 0) {
    if (workspace == nullptr || workspace_bytes < norm_partials_bytes(M, norm_groups, norm_width))
      return WDIT_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return WDIT_ERR_ALIGN;
  }
  return run_norm(A, lda, B, ldb, out, ldo, M, N, K, vec, ln_csum, ln_stats, ln_stats_tiles, ln_stats_width, ln_eps,
                  norm_groups, norm_width, norm_w0, norm_w1, norm_eps, rope_groups, rope_cos, rope_sin, rope_ld,
                  rows_per_batch, token_offset, static_cast<float*>(workspace), static_cast<cudaStream_t>(stream),
                  max_ctas);
}

int wdit_gemm_norm_fused(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                         const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                         int ln_stats_width, float ln_eps, int norm_groups, int norm_width, const float* norm_w0,
                         const float* norm_w1, float norm_eps, int rope_groups, const float* rope_cos,
                         const float* rope_sin, int rope_ld, int rows_per_batch, int token_offset, void* stream,
                         int max_ctas) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (norm_groups < 1) return WDIT_ERR_ARG;
  int rc = check_norm(A, lda, B, ldb, out, ldo, M, N, K, vec, norm_groups, norm_width, norm_w0, norm_w1, rope_groups,
                      rope_cos, rope_sin, rope_ld, rows_per_batch, token_offset);
  if (rc) return rc;
  if (norm_width % BN != 0) return WDIT_ERR_SHAPE;  // units are whole N tiles
  return run_norm_fused(A, lda, B, ldb, out, ldo, M, N, K, vec, ln_csum, ln_stats, ln_stats_tiles, ln_stats_width,
                        ln_eps, norm_groups, norm_width, norm_w0, norm_w1, norm_eps, rope_groups, rope_cos, rope_sin,
                        rope_ld, rows_per_batch, token_offset, static_cast<cudaStream_t>(stream), max_ctas);
}

int wdit_gemm_norm_exchange(const void* A, int lda, const void* B, int ldb, void* qk_scratch, int ld_scratch, int M,
                            int K, const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                            int ln_stats_width, float ln_eps, const float* wq, const float* wk, float eps,
                            const float* rope_cos, const float* rope_sin, int rope_ld, int batch, int Lp, int H,
                            int P, int rank, const void* const* peer_bases, long long full_off, long long flag_off,
                            unsigned int epoch, unsigned int* done_ctr, void* stream, int max_ctas) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (peer_bases == nullptr || done_ctr == nullptr || qk_scratch == nullptr) return WDIT_ERR_ARG;
  if (H <= 0 || batch <= 0 || Lp <= 0 || P < 1 || P > kXchgMaxPeers || rank < 0 || rank >= P ||
      (batch * H) % P != 0 || batch * Lp != M)
    return WDIT_ERR_SHAPE;
  const int D = H * 128;
  const int N = 3 * D;
  if (ld_scratch < N) return WDIT_ERR_SHAPE;
  int rc = check_norm(A, lda, B, ldb, qk_scratch, ld_scratch, M, N, K, vec, 2, D, wq, wk, 2, rope_cos, rope_sin,
                      rope_ld, Lp, rank * Lp);
  if (rc) return rc;
  if (D % BN != 0) return WDIT_ERR_SHAPE;
  if ((full_off & 255) != 0 || (flag_off & 255) != 0) return WDIT_ERR_ALIGN;
  XchgParams xc = {};
  for (int q = 0; q < P; ++q) {
    if (peer_bases[q] == nullptr || (reinterpret_cast<uintptr_t>(peer_bases[q]) & 255) != 0) return WDIT_ERR_ALIGN;
    xc.base[q] = static_cast<unsigned char*>(const_cast<void*>(peer_bases[q]));
  }
  xc.full_off = full_off;
  xc.flag_off = flag_off;
  xc.done_ctr = done_ctr;
  xc.epoch = epoch;
  xc.P = P;
  xc.rank = rank;
  xc.B = batch;
  xc.Lp = Lp;
  xc.H = H;
  xc.U = batch * H / P;
  xc.L = P * Lp;
  return run_norm_fused(A, lda, B, ldb, qk_scratch, ld_scratch, M, N, K, vec, ln_csum, ln_stats, ln_stats_tiles,
                        ln_stats_width, ln_eps, 2, D, wq, wk, eps, 2, rope_cos, rope_sin, rope_ld, Lp, rank * Lp,
                        static_cast<cudaStream_t>(stream), max_ctas, &xc);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of wdit_gemm_norm.
//
// Some callers cannot allocate device memory at the point where they run this GEMM: code
// that executes inside a region where allocation is not permitted (for example while
// another component is recording work for replay, or inside a fixed memory budget that
// was reserved up front), and hosts whose allocator is owned by a different runtime and
// is not reachable from the call site. For them the RMSNorm partials live in a fixed,
// file-scope device array instead of a caller-supplied workspace.
//
// Limits and sharing rules:
//   * The array holds WDIT_STATIC_SCRATCH_BYTES (4 MiB) on every GPU that loads this
//     library, for the lifetime of the process.
//   * A call needs wdit_gemm_norm_workspace_bytes(M, N, norm_groups, norm_width) bytes of
//     it; larger problems are rejected with WDIT_ERR_SCRATCH_LIMIT before any launch.
//   * All calls on a device share the one array; calls that overlap on the GPU (different
//     streams with no ordering between them) race on it.
//   * The first call on a device looks the array's device address up once
//     (cudaGetSymbolAddress, with that device current); make that first call before any
//     stream capture begins.
// ---------------------------------------------------------------------------
namespace wdit {
namespace {

static __device__ __align__(256) unsigned char g_norm_static_scratch[WDIT_STATIC_SCRATCH_BYTES];

std::mutex g_static_scratch_mutex;
void* g_static_scratch_addr[64] = {};

// Device address of the static scratch on the current device (looked up once per device).
int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
  if (dev < 0 || dev >= 64) return WDIT_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_addr[dev] == nullptr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_norm_static_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();  // the lookup's error is not sticky: do not leave it for a later launch check
      return WDIT_ERR_CUDA_BASE + static_cast<int>(e);
    }
    if (addr == nullptr) return WDIT_ERR_ARG;
    g_static_scratch_addr[dev] = addr;
  }
  *out = g_static_scratch_addr[dev];
  return WDIT_OK;
}

}  // namespace
}  // namespace wdit

extern "C" {

long long wdit_static_scratch_bytes(void) { return WDIT_STATIC_SCRATCH_BYTES; }

int wdit_gemm_norm_static(const void* A, int lda, const void* B, int ldb, void* out, int ldo, int M, int N, int K,
                          const float* vec, const float* ln_csum, const float* ln_stats, int ln_stats_tiles,
                          int ln_stats_width, float ln_eps, int norm_groups, int norm_width, const float* norm_w0,
                          const float* norm_w1, float norm_eps, int rope_groups, const float* rope_cos,
                          const float* rope_sin, int rope_ld, int rows_per_batch, int token_offset, void* stream,
                          int max_ctas) {
  if (M == 0) return WDIT_OK;  // no rows: nothing to do (pointers are not looked at)
  if (norm_groups < 1) return WDIT_ERR_ARG;
  int rc = check_norm(A, lda, B, ldb, out, ldo, M, N, K, vec, norm_groups, norm_width, norm_w0, norm_w1, rope_groups,
                      rope_cos, rope_sin, rope_ld, rows_per_batch, token_offset);
  if (rc) return rc;
  if (norm_partials_bytes(M, norm_groups, norm_width) > static_cast<long long>(WDIT_STATIC_SCRATCH_BYTES))
    return WDIT_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if ((rc = static_scratch_address(&scratch))) return rc;
  return run_norm(A, lda, B, ldb, out, ldo, M, N, K, vec, ln_csum, ln_stats, ln_stats_tiles, ln_stats_width, ln_eps,
                  norm_groups, norm_width, norm_w0, norm_w1, norm_eps, rope_groups, rope_cos, rope_sin, rope_ld,
                  rows_per_batch, token_offset, static_cast<float*>(scratch), static_cast<cudaStream_t>(stream),
                  max_ctas);
}

}  // extern "C"
