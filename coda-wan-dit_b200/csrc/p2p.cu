// Ulysses all-to-all of the token-sharded forward as direct NVLink stores between peer GPUs.
//
// Rank r of P owns tokens [r*Lp, (r+1)*Lp) of each of the B batch entries; self-attention
// needs every token of a (batch, head) unit u = b*H + h, and unit u lives on rank u / U
// (U = B*H/P units per rank). Each rank exposes one "exchange region" of its own memory to
// its peers (CUDA IPC, mapped once):
//
//   full[2][3][U][L][hd]   bf16  q, k, v of this rank's units, all L = P*Lp tokens
//   y[2][B*Lp][D]          bf16  attention output rows of this rank's tokens (D = H*hd)
//   flags[2][P]            u32   arrival epochs: flags[x][s] = last epoch in which rank s
//                                completed its writes of exchange x into this region
//
// Exchange 1 (p2p_qkv_kernel): one warp per local row reads the QKV GEMM output, applies the
// full-width q/k RMSNorm (from the GEMM's per-128-column mean-square partials) and 3D RoPE,
// and stores every 128-column head straight into full[buf] of the rank owning that unit, at
// the row's global token position. This fuses the RMSNorm/RoPE pass, the send-buffer pack,
// the all-to-all and the receive-side gather into one pass over the data.
// Exchange 2 (p2p_out_kernel): the attention output o[U][L][hd] of this rank's units goes
// back, one 256-byte head row per token, into y[buf] of the rank owning the token.
//
// Completion: every thread fences its stores at system scope, the block counts itself done
// on a local counter, and the last block of the grid publishes `epoch` into flags[x][r] of
// every rank with a system-scope release store. p2p_wait_kernel polls this rank's flags with
// acquire loads until all P ranks have published the epoch (bounded by the library's wait
// limit; on expiry it records a timeout in the error record and returns).
// Double buffering by epoch parity makes a "buffer free" handshake unnecessary: a rank can
// write buffer (e & 1) of a peer only after consuming data the peer produced after it had
// finished with that buffer's previous contents (epoch e - 2).
//
// No TMA and no multicast: plain 16-byte ld/st through the peer mappings.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "wdit_internal.h"

namespace wdit {
namespace {

constexpr int kMaxPeers = 8;
constexpr int kP2PWarps = 8;     // rows (or token pairs) per block iteration
constexpr int kVecPerPass = 6;   // 16-byte vectors per lane loaded before storing (1536 columns)
constexpr unsigned int kErrTimeoutCode = 0x7117u;
constexpr unsigned int kSiteP2PWait = 9;

struct PeerTable {
  unsigned char* base[kMaxPeers];  // exchange region of each rank, as mapped in this process
};

__device__ __forceinline__ uint64_t gtimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_v4(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// All stores of this block are complete system-wide; the last block of the grid publishes
// `epoch` to flags[r] of every rank and resets the local completion counter.
__device__ __forceinline__ void publish_done(const PeerTable& peers, int P, int my_rank, long long flag_off,
                                             unsigned int epoch, unsigned int* done_ctr) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int old = atomicAdd(done_ctr, 1u);
    if (old == gridDim.x - 1) {
      __threadfence_system();
      for (int p = 0; p < P; ++p) {
        st_release_sys(reinterpret_cast<unsigned int*>(peers.base[p] + flag_off) + my_rank, epoch);
      }
      atomicExch(done_ctr, 0u);
    }
  }
}

// One warp per local row (b, t): q and k get WanRMSNorm + RoPE, v is copied; every 128-column
// head goes to full[m][u % U][r*Lp + t] of rank u / U.
__global__ void __launch_bounds__(32 * kP2PWarps)
    p2p_qkv_kernel(const __nv_bfloat16* __restrict__ qkv, int ldq, const float* __restrict__ part, int part_ld,
                   const float* __restrict__ wq, const float* __restrict__ wk, float eps,
                   const float* __restrict__ cs, const float* __restrict__ sn, int rope_ld, int B, int Lp, int H,
                   int P, int my_rank, const __grid_constant__ PeerTable peers, long long full_off, long long flag_off, unsigned int epoch,
                   unsigned int* done_ctr) {
  constexpr int hd = 128;
  const int lane = threadIdx.x & 31;
  const int D = H * hd;
  const int U = B * H / P;
  const int L = P * Lp;
  const int rows = B * Lp;
  const int parts = D / 128;
  for (int row = blockIdx.x * kP2PWarps + (threadIdx.x >> 5); row < rows; row += gridDim.x * kP2PWarps) {
    const int b = row / Lp;
    const int t = row - b * Lp;
    const __nv_bfloat16* src = qkv + static_cast<size_t>(row) * ldq;
    const float* pr = part + static_cast<size_t>(row) * part_ld;
    float msq = 0.f, msk = 0.f;
    for (int j = lane; j < parts; j += 32) {
      msq += pr[j];
      msk += pr[parts + j];
    }
    const size_t tok = static_cast<size_t>(my_rank) * Lp + t;  // global token index
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + tok * rope_ld) + (lane & 15));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(sn + tok * rope_ld) + (lane & 15));
    const float rq = rsqrtf(warp_sum(msq) / static_cast<float>(parts) + eps);
    const float rk = rsqrtf(warp_sum(msk) / static_cast<float>(parts) + eps);
    const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
    const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
    for (int m = 0; m < 3; ++m) {
      const float* w = m == 0 ? wq : wk;
      const float rstd = m == 0 ? rq : rk;
      for (int c0 = lane * 8; c0 < D; c0 += kVecPerPass * 256) {
        // All of this pass's loads are issued before the first store.
        uint4 vin[kVecPerPass];
#pragma unroll
        for (int j = 0; j < kVecPerPass; ++j) {
          if (c0 + j * 256 < D) vin[j] = ld_v4(src + m * D + c0 + j * 256);
        }
#pragma unroll
        for (int j = 0; j < kVecPerPass; ++j) {
          const int c = c0 + j * 256;
          if (c >= D) break;
          uint4 raw = vin[j];
          if (m < 2) {
            const float4 wa = __ldg(reinterpret_cast<const float4*>(w + c));
            const float4 wb = __ldg(reinterpret_cast<const float4*>(w + c + 4));
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
            uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
            float v[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              v[2 * i] = __uint_as_float(rw[i] << 16);
              v[2 * i + 1] = __uint_as_float(rw[i] & 0xFFFF0000u);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = bf16r(bf16r(v[i] * rstd) * wv[i]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float e = v[2 * i], o = v[2 * i + 1];
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(e * cc[i] - o * ss[i], e * ss[i] + o * cc[i]);
              rw[i] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            raw = make_uint4(rw[0], rw[1], rw[2], rw[3]);
          }
          const int h = c / hd;
          const int u = b * H + h;
          const int p = u / U;
          const int ul = u - p * U;
          unsigned char* dst = peers.base[p] + full_off +
                               ((((static_cast<long long>(m) * U + ul) * L + tok) * hd + (c - h * hd)) * 2);
          st_v4(dst, raw);
        }
      }
    }
  }
  publish_done(peers, P, my_rank, flag_off, epoch, done_ctr);
}

// o[ul][g][0:hd] (this rank's unit ul = u % U, global token g) -> y[b*Lp + t][h*hd ...] of
// rank g / Lp. One warp moves two tokens (16 lanes x 16 bytes each).
__global__ void __launch_bounds__(32 * kP2PWarps)
    p2p_out_kernel(const __nv_bfloat16* __restrict__ o, long long o_su, long long o_st, int B, int Lp, int H,
                   int P, int my_rank, const __grid_constant__ PeerTable peers, long long y_off, int ldy, long long flag_off,
                   unsigned int epoch, unsigned int* done_ctr) {
  constexpr int hd = 128;
  const int lane = threadIdx.x & 31;
  const int U = B * H / P;
  const int L = P * Lp;
  const long long pairs = static_cast<long long>(U) * L / 2;  // L even: checked on the host
  for (long long it = static_cast<long long>(blockIdx.x) * kP2PWarps + (threadIdx.x >> 5); it < pairs;
       it += static_cast<long long>(gridDim.x) * kP2PWarps) {
    const long long flat = it * 2 + (lane >> 4);
    const int ul = static_cast<int>(flat / L);
    const int g = static_cast<int>(flat - static_cast<long long>(ul) * L);
    const int col = (lane & 15) * 8;
    const uint4 raw = ld_v4(o + ul * o_su + static_cast<long long>(g) * o_st + col);
    const int u = my_rank * U + ul;
    const int b = u / H;
    const int h = u - b * H;
    const int p = g / Lp;
    const int t = g - p * Lp;
    unsigned char* dst =
        peers.base[p] + y_off + ((static_cast<long long>(b) * Lp + t) * ldy + static_cast<long long>(h) * hd + col) * 2;
    st_v4(dst, raw);
  }
  publish_done(peers, P, my_rank, flag_off, epoch, done_ctr);
}

// Wait until every rank has published `epoch` for this exchange (bounded).
__global__ void p2p_wait_kernel(const unsigned int* flags, int P, unsigned int epoch, unsigned long long limit_ns,
                                unsigned int* err) {
  const int lane = threadIdx.x;
  bool ok = true;
  if (lane < P) {
    const unsigned int* f = flags + lane;
    if (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
      const uint64_t t0 = gtimer_ns();
      while (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
        if (gtimer_ns() - t0 > limit_ns) {
          ok = false;
          break;
        }
        __nanosleep(100);
      }
    }
  }
  if (!ok && err != nullptr && atomicCAS(err, 0u, kErrTimeoutCode) == 0u) {
    err[1] = kSiteP2PWait;
    err[2] = static_cast<unsigned int>(lane);  // rank that did not arrive
    err[3] = epoch;
    __threadfence();
  }
}

inline int status_of(cudaError_t e) { return e == cudaSuccess ? WDIT_OK : WDIT_ERR_CUDA_BASE + static_cast<int>(e); }

int p2p_grid() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms * 4;
}

bool fill_peers(PeerTable* t, const void* const* bases, int P) {
  if (P < 1 || P > kMaxPeers) return false;
  memset(t, 0, sizeof(*t));
  for (int p = 0; p < P; ++p) {
    if (bases[p] == nullptr || (reinterpret_cast<uintptr_t>(bases[p]) & 255) != 0) return false;
    t->base[p] = static_cast<unsigned char*>(const_cast<void*>(bases[p]));
  }
  return true;
}

PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;
std::once_flag g_addr_range_once;

}  // namespace
}  // namespace wdit

using namespace wdit;

extern "C" {

int wdit_ipc_handle(const void* ptr, void* handle_out, long long* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return WDIT_ERR_ARG;
  std::call_once(g_addr_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (g_addr_range == nullptr) return WDIT_ERR_DRIVER;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return WDIT_ERR_DRIVER;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return status_of(e);
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<long long>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return WDIT_OK;
}

int wdit_ipc_open(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr) return WDIT_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return status_of(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
}

int wdit_ipc_close(void* base) {
  if (base == nullptr) return WDIT_ERR_ARG;
  return status_of(cudaIpcCloseMemHandle(base));
}

int wdit_p2p_qkv_exchange(const void* qkv, int ldq, const float* part, int part_ld, const float* wq,
                          const float* wk, float eps, const float* rope_cos, const float* rope_sin, int rope_ld,
                          int B, int Lp, int H, int hd, int P, int rank, const void* const* peer_bases,
                          long long full_off, long long flag_off, unsigned int epoch, unsigned int* done_ctr,
                          void* stream) {
  if (qkv == nullptr || part == nullptr || wq == nullptr || wk == nullptr || rope_cos == nullptr ||
      rope_sin == nullptr || peer_bases == nullptr || done_ctr == nullptr)
    return WDIT_ERR_ARG;
  if (hd != 128 || B <= 0 || Lp <= 0 || H <= 0 || P < 1 || P > kMaxPeers || rank < 0 || rank >= P ||
      (B * H) % P != 0 || ldq < 3 * H * hd || part_ld < 2 * H || rope_ld < 64)
    return WDIT_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || ldq % 8 || (reinterpret_cast<uintptr_t>(wq) & 15) ||
      (reinterpret_cast<uintptr_t>(wk) & 15) || (reinterpret_cast<uintptr_t>(rope_cos) & 15) ||
      (reinterpret_cast<uintptr_t>(rope_sin) & 15) || rope_ld % 4 || (full_off & 255) || (flag_off & 255))
    return WDIT_ERR_ALIGN;
  PeerTable peers;
  if (!fill_peers(&peers, peer_bases, P)) return WDIT_ERR_ARG;
  const int rows = B * Lp;
  int grid = p2p_grid();
  const int need = (rows + kP2PWarps - 1) / kP2PWarps;
  if (need < grid) grid = need;
  p2p_qkv_kernel<<<grid, 32 * kP2PWarps, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), ldq, part, part_ld, wq, wk, eps, rope_cos, rope_sin, rope_ld, B, Lp, H,
      P, rank, peers, full_off, flag_off, epoch, done_ctr);
  return status_of(cudaGetLastError());
}

int wdit_p2p_out_exchange(const void* o, long long o_unit_stride, long long o_tok_stride, int B, int Lp, int H,
                          int hd, int P, int rank, const void* const* peer_bases, long long y_off, int ldy,
                          long long flag_off, unsigned int epoch, unsigned int* done_ctr, void* stream) {
  if (o == nullptr || peer_bases == nullptr || done_ctr == nullptr) return WDIT_ERR_ARG;
  if (hd != 128 || B <= 0 || Lp <= 0 || H <= 0 || P < 1 || P > kMaxPeers || rank < 0 || rank >= P ||
      (B * H) % P != 0 || ldy < H * hd || (P * Lp) % 2 != 0)
    return WDIT_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(o) & 15) || o_unit_stride % 8 || o_tok_stride % 8 || ldy % 8 || (y_off & 255) ||
      (flag_off & 255))
    return WDIT_ERR_ALIGN;
  PeerTable peers;
  if (!fill_peers(&peers, peer_bases, P)) return WDIT_ERR_ARG;
  const long long pairs = static_cast<long long>(B * H / P) * P * Lp / 2;
  int grid = p2p_grid();
  const long long need = (pairs + kP2PWarps - 1) / kP2PWarps;
  if (need < grid) grid = static_cast<int>(need);
  p2p_out_kernel<<<grid, 32 * kP2PWarps, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(o), o_unit_stride, o_tok_stride, B, Lp, H, P, rank, peers, y_off, ldy,
      flag_off, epoch, done_ctr);
  return status_of(cudaGetLastError());
}

int wdit_p2p_wait(const unsigned int* flags, int P, unsigned int epoch, void* stream) {
  if (flags == nullptr) return WDIT_ERR_ARG;
  if (P < 1 || P > 32) return WDIT_ERR_SHAPE;
  unsigned int* err = nullptr;
  int rc = error_record_ptr(&err);
  if (rc) return rc;
  p2p_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, P, epoch, wait_limit_ns(), err);
  return status_of(cudaGetLastError());
}

}  // extern "C"
