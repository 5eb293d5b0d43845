// Layout kernels for the Ulysses all-to-all around self-attention, and small helpers.
//
// Sequence parallelism: rank r owns tokens [r*Lp, (r+1)*Lp) of every batch entry
// (Lp = L / P) and all heads. Attention needs all L tokens of a head, so the B*H
// (batch, head) pairs are dealt out as "units": unit u = b*H + h belongs to rank
// u / U with U = B*H / P units per rank. This divides evenly for Wan-1.3B's 12 heads
// at P = 8 with CFG batch 2 (24 units, 3 per rank), which plain head sharding cannot.
//
//   ulysses_pack     token-sharded rows  [B*Lp, ld] (nmat column blocks of H*hd)
//                    -> send[P][nmat][U][Lp][hd]          (before the all-to-all)
//   seq_gather       recv[P][nmat][U][Lp][hd] -> attn[nmat][U][P*Lp][hd]
//   seq_scatter      attention output o(u, token) (strided) -> send[P][U][Lp][hd]
//   ulysses_unpack   recv[P][U][Lp][hd] -> token-sharded rows [B*Lp, ld]
// All copies move 16-byte vectors of bf16 (hd % 8 == 0); one thread per vector.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "wdit_internal.h"

namespace wdit {
namespace {

inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WDIT_OK : WDIT_ERR_CUDA_BASE + static_cast<int>(e);
}

inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline unsigned blocks_for(long long n) { return static_cast<unsigned>((n + 255) / 256); }

__global__ void ulysses_pack_kernel(const uint4* __restrict__ src, long long ld_v, int B, int Lp, int H, int hdv,
                                    int nmat, int P, uint4* __restrict__ dst) {
  // dst index: ((((d * nmat + c) * U + j) * Lp + t) * hdv + v)
  const int U = B * H / P;
  const long long total = static_cast<long long>(P) * nmat * U * Lp * hdv;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  long long q = i;
  const int v = static_cast<int>(q % hdv);
  q /= hdv;
  const int t = static_cast<int>(q % Lp);
  q /= Lp;
  const int j = static_cast<int>(q % U);
  q /= U;
  const int c = static_cast<int>(q % nmat);
  const int d = static_cast<int>(q / nmat);
  const int u = d * U + j;
  const int b = u / H;
  const int h = u - b * H;
  dst[i] = src[(static_cast<long long>(b) * Lp + t) * ld_v + (static_cast<long long>(c) * H + h) * hdv + v];
}

__global__ void seq_gather_kernel(const uint4* __restrict__ recv, int nmat, int U, int P, int Lp, int hdv,
                                  uint4* __restrict__ dst) {
  // dst index: (((c * U + j) * (P * Lp) + s * Lp + t) * hdv + v)
  const long long total = static_cast<long long>(P) * nmat * U * Lp * hdv;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  long long q = i;
  const int v = static_cast<int>(q % hdv);
  q /= hdv;
  const long long L = static_cast<long long>(P) * Lp;
  const long long tok = q % L;
  q /= L;
  const int j = static_cast<int>(q % U);
  const int c = static_cast<int>(q / U);
  const int s = static_cast<int>(tok / Lp);
  const int t = static_cast<int>(tok - static_cast<long long>(s) * Lp);
  dst[i] = recv[((((static_cast<long long>(s) * nmat + c) * U + j) * Lp + t) * hdv) + v];
}

__global__ void seq_scatter_kernel(const uint4* __restrict__ o, long long unit_stride_v, long long tok_stride_v, int U,
                                   int P, int Lp, int hdv, uint4* __restrict__ dst) {
  // dst index: (((s * U + j) * Lp + t) * hdv + v); source token = s * Lp + t of unit j
  const long long total = static_cast<long long>(P) * U * Lp * hdv;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  long long q = i;
  const int v = static_cast<int>(q % hdv);
  q /= hdv;
  const int t = static_cast<int>(q % Lp);
  q /= Lp;
  const int j = static_cast<int>(q % U);
  const int s = static_cast<int>(q / U);
  dst[i] = o[static_cast<long long>(j) * unit_stride_v + (static_cast<long long>(s) * Lp + t) * tok_stride_v + v];
}

__global__ void ulysses_unpack_kernel(const uint4* __restrict__ recv, int B, int Lp, int H, int hdv, int P,
                                      uint4* __restrict__ dst, long long ld_v) {
  // dst index: ((b * Lp + t) row, (h * hdv + v) vector column)
  const int U = B * H / P;
  const long long total = static_cast<long long>(B) * Lp * H * hdv;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  long long q = i;
  const int v = static_cast<int>(q % hdv);
  q /= hdv;
  const int h = static_cast<int>(q % H);
  q /= H;
  const int t = static_cast<int>(q % Lp);
  const int b = static_cast<int>(q / Lp);
  const int u = b * H + h;
  const int d = u / U;
  const int j = u - d * U;
  dst[(static_cast<long long>(b) * Lp + t) * ld_v + static_cast<long long>(h) * hdv + v] =
      recv[((static_cast<long long>(d) * U + j) * Lp + t) * hdv + v];
}

}  // namespace
}  // namespace wdit

using namespace wdit;

extern "C" {

int wdit_set_device(int device) {
  const cudaError_t e = cudaSetDevice(device);
  return e == cudaSuccess ? WDIT_OK : WDIT_ERR_CUDA_BASE + static_cast<int>(e);
}

int wdit_ulysses_pack(const void* src, int ld, int B, int Lp, int H, int hd, int nmat, int P, void* send,
                      void* stream) {
  if (src == nullptr || send == nullptr) return WDIT_ERR_ARG;
  if (B <= 0 || Lp <= 0 || H <= 0 || P <= 0 || nmat <= 0 || hd % 8 != 0 || (B * H) % P != 0) return WDIT_ERR_SHAPE;
  if (ld < nmat * H * hd || ld % 8 != 0) return WDIT_ERR_SHAPE;
  if (!a16(src) || !a16(send)) return WDIT_ERR_ALIGN;
  const long long total = static_cast<long long>(B) * Lp * H * nmat * (hd / 8);
  ulysses_pack_kernel<<<blocks_for(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), ld / 8, B, Lp, H, hd / 8, nmat, P, static_cast<uint4*>(send));
  return launch_status();
}

int wdit_seq_gather(const void* recv, int nmat, int U, int P, int Lp, int hd, void* dst, void* stream) {
  if (recv == nullptr || dst == nullptr) return WDIT_ERR_ARG;
  if (nmat <= 0 || U <= 0 || P <= 0 || Lp <= 0 || hd % 8 != 0) return WDIT_ERR_SHAPE;
  if (!a16(recv) || !a16(dst)) return WDIT_ERR_ALIGN;
  const long long total = static_cast<long long>(P) * nmat * U * Lp * (hd / 8);
  seq_gather_kernel<<<blocks_for(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(recv), nmat, U, P, Lp, hd / 8, static_cast<uint4*>(dst));
  return launch_status();
}

int wdit_seq_scatter(const void* o, long long unit_stride, long long tok_stride, int U, int P, int Lp, int hd,
                     void* send, void* stream) {
  if (o == nullptr || send == nullptr) return WDIT_ERR_ARG;
  if (U <= 0 || P <= 0 || Lp <= 0 || hd % 8 != 0) return WDIT_ERR_SHAPE;
  if (unit_stride % 8 != 0 || tok_stride % 8 != 0 || !a16(o) || !a16(send)) return WDIT_ERR_ALIGN;
  const long long total = static_cast<long long>(P) * U * Lp * (hd / 8);
  seq_scatter_kernel<<<blocks_for(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(o), unit_stride / 8, tok_stride / 8, U, P, Lp, hd / 8, static_cast<uint4*>(send));
  return launch_status();
}

int wdit_ulysses_unpack(const void* recv, int B, int Lp, int H, int hd, int P, void* dst, int ld, void* stream) {
  if (recv == nullptr || dst == nullptr) return WDIT_ERR_ARG;
  if (B <= 0 || Lp <= 0 || H <= 0 || P <= 0 || hd % 8 != 0 || (B * H) % P != 0) return WDIT_ERR_SHAPE;
  if (ld < H * hd || ld % 8 != 0) return WDIT_ERR_SHAPE;
  if (!a16(recv) || !a16(dst)) return WDIT_ERR_ALIGN;
  const long long total = static_cast<long long>(B) * Lp * H * (hd / 8);
  ulysses_unpack_kernel<<<blocks_for(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(recv), B, Lp, H, hd / 8, P, static_cast<uint4*>(dst), ld / 8);
  return launch_status();
}

}  // extern "C"
