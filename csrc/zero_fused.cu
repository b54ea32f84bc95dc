// Fused ZeRO optimizer collectives over NVLink peer memory.
//
//  reduce-scatter: every rank has packed its flat gradient (bf16 or fp32) into its symmetric staging buffer and the
//                  ranks have exchanged "ready" flags. Rank r then sums elements [start, start + per) of all ranks'
//                  buffers with peer loads in a fixed rank order (deterministic), scales by 1/world, writes its fp32
//                  shard gradient and per-block sums of squares (for the global clip norm). This replaces
//                  reduce_scatter + the cast and scale kernels.
//  update+gather:  AdamW on the shard (fp32 master and moments, clip coefficient read on the device), then the new
//                  value (cast to the parameter dtype) is stored into EVERY rank's flat parameter buffer at the same
//                  position. The replicated parameters live in those symmetric buffers, so this store is the
//                  all-gather: no separate collective and no unpack copy. Ranks exchange "done" flags afterwards.
// Only plain loads and stores to peer memory; flags use the release/acquire kernels of ep_fused.cu / p2p.cu.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

__device__ __forceinline__ float load_any(const void* base, int64_t i, int dtype) {
  return dtype == 0 ? static_cast<const float*>(base)[i] : __bfloat162float(static_cast<const bf16*>(base)[i]);
}

__global__ void __launch_bounds__(256) zero_rs_kernel(const void* const* __restrict__ peers, int world, int dtype,
                                                      int64_t start, int64_t per, float inv_world,
                                                      float* __restrict__ shard, double* __restrict__ partial) {
  float sq = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += load_any(peers[r], start + i, dtype);  // NVLink loads, fixed order
    s *= inv_world;
    shard[i] = s;
    sq += s * s;
  }
  __shared__ float red[8];
  sq = warp_sum(sq);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    double acc = 0.0;
    for (int w = 0; w < blockDim.x / 32; ++w) acc += red[w];
    partial[blockIdx.x] = acc;
  }
}

__global__ void __launch_bounds__(256) zero_adamw_gather_kernel(float* __restrict__ master, float* __restrict__ m,
                                                                float* __restrict__ v,
                                                                const float* __restrict__ grad,
                                                                const float* __restrict__ clip, AdamHyper h,
                                                                void* const* __restrict__ peers, int world,
                                                                int dtype, int64_t start, int64_t per,
                                                                int64_t valid) {
  const float coef = clip ? clip[0] : 1.f;
  const float decay = 1.f - h.lr * h.weight_decay;
  const float step_size = h.lr / h.bias_correction1;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (start + i >= valid) break;  // padding past the last parameter
    const float g = grad[i] * coef;
    float p = master[i] * decay;
    const float mm = h.beta1 * m[i] + (1.f - h.beta1) * g;
    const float vv = h.beta2 * v[i] + (1.f - h.beta2) * g * g;
    p -= step_size * mm / (sqrtf(vv) / h.bias_correction2_sqrt + h.eps);
    master[i] = p;
    m[i] = mm;
    v[i] = vv;
    for (int r = 0; r < world; ++r) {  // NVLink stores: the all-gather
      if (dtype == 0) static_cast<float*>(peers[r])[start + i] = p;
      else static_cast<bf16*>(peers[r])[start + i] = __float2bfloat16(p);
    }
  }
}

}  // namespace

int zero_rs_blocks(int64_t per) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(592, (per + 255) / 256))); }

void zero_reduce_scatter(const void* const* peers, int world, int dtype, int64_t start, int64_t per, float* shard,
                         double* partial, cudaStream_t stream) {
  if (per == 0) return;
  zero_rs_kernel<<<zero_rs_blocks(per), 256, 0, stream>>>(peers, world, dtype, start, per, 1.f / world, shard,
                                                          partial);
  check_cuda(cudaGetLastError(), "zero_reduce_scatter");
}

void zero_adamw_gather(float* master, float* m, float* v, const float* grad, const float* clip, const AdamHyper& h,
                       void* const* peers, int world, int dtype, int64_t start, int64_t per, int64_t valid,
                       cudaStream_t stream) {
  if (per == 0) return;
  zero_adamw_gather_kernel<<<zero_rs_blocks(per), 256, 0, stream>>>(master, m, v, grad, clip, h, peers, world, dtype,
                                                                    start, per, valid);
  check_cuda(cudaGetLastError(), "zero_adamw_gather");
}

}  // namespace qw
