// Tensor-parallel all-reduce fused with the producing GEMM (row-parallel output projection forward; column-parallel
// input projection backward).
//
// The GEMM epilogue (gemm_tcgen05.cuh, `peer_out`) has already stored this rank's partial rows into the owning
// ranks' staging buffers over NVLink: rank r's staging holds [world][rows_per_rank][N], slot s = rank s's partial of
// rows [r*rows_per_rank, (r+1)*rows_per_rank). After the ready barrier, rank r sums its rows over the slots in a fixed
// rank order (deterministic, fp32), adds the replicated bias, and stores the result into every rank's output buffer
// at the same rows — the all-gather half — so each rank ends with the full reduced [M, N]. Plain peer loads/stores
// only; the barriers around it are the release/acquire flag kernels of ep_fused.cu / p2p.cu.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

__global__ void __launch_bounds__(256) tp_reduce_bcast_kernel(const bf16* __restrict__ staging, int world,
                                                              int64_t rows, int N, const float* __restrict__ bias,
                                                              void* const* __restrict__ outs, int me) {
  const int vec_per_row = N / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx / vec_per_row;
    const int c = static_cast<int>(idx % vec_per_row) * 8;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = bias ? bias[c + j] : 0.f;
    for (int s = 0; s < world; ++s) {
      const uint4 v = *reinterpret_cast<const uint4*>(staging + (static_cast<int64_t>(s) * rows + i) * N + c);
      const bf16* b = reinterpret_cast<const bf16*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(b[j]);
    }
    uint4 w;
    w.x = pack_bf16(acc[0], acc[1]);
    w.y = pack_bf16(acc[2], acc[3]);
    w.z = pack_bf16(acc[4], acc[5]);
    w.w = pack_bf16(acc[6], acc[7]);
    const int64_t off = (static_cast<int64_t>(me) * rows + i) * N + c;
    for (int r = 0; r < world; ++r) *reinterpret_cast<uint4*>(static_cast<bf16*>(outs[r]) + off) = w;  // NVLink
  }
}

// out[i] = bias + sum over slots s (fixed order) of staging[s][i]: this rank's rows of a reduce-scatter whose partial
// rows the producing GEMM already stored into the staging slots
__global__ void __launch_bounds__(256) tp_reduce_rows_kernel(const bf16* __restrict__ staging, int world,
                                                             int64_t rows, int N, const float* __restrict__ bias,
                                                             bf16* __restrict__ out) {
  const int vec_per_row = N / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx / vec_per_row;
    const int c = static_cast<int>(idx % vec_per_row) * 8;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = bias ? bias[c + j] : 0.f;
    for (int s = 0; s < world; ++s) {
      const uint4 v = *reinterpret_cast<const uint4*>(staging + (static_cast<int64_t>(s) * rows + i) * N + c);
      const bf16* b = reinterpret_cast<const bf16*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(b[j]);
    }
    uint4 w;
    w.x = pack_bf16(acc[0], acc[1]);
    w.y = pack_bf16(acc[2], acc[3]);
    w.z = pack_bf16(acc[4], acc[5]);
    w.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + i * N + c) = w;
  }
}

}  // namespace

void tp_reduce_rows(const bf16* staging, int world, int64_t rows_per_rank, int N, const float* bias, bf16* out,
                    cudaStream_t stream) {
  if (rows_per_rank == 0 || N == 0) return;
  if (N % 8) throw std::runtime_error("tp_reduce_rows: N must be a multiple of 8");
  const int64_t total = rows_per_rank * (N / 8);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(148 * 8, (total + 255) / 256)));
  tp_reduce_rows_kernel<<<grid, 256, 0, stream>>>(staging, world, rows_per_rank, N, bias, out);
  check_cuda(cudaGetLastError(), "tp_reduce_rows");
}

void tp_reduce_bcast(const bf16* staging, int world, int64_t rows_per_rank, int N, const float* bias,
                     void* const* outs, int me, cudaStream_t stream) {
  if (rows_per_rank == 0 || N == 0) return;
  if (N % 8) throw std::runtime_error("tp_reduce_bcast: N must be a multiple of 8");
  const int64_t total = rows_per_rank * (N / 8);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(148 * 8, (total + 255) / 256)));
  tp_reduce_bcast_kernel<<<grid, 256, 0, stream>>>(staging, world, rows_per_rank, N, bias, outs, me);
  check_cuda(cudaGetLastError(), "tp_reduce_bcast");
}

int tp_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
