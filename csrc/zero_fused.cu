// Fused ZeRO optimizer collectives over NVLink peer memory.
//
//  reduce-scatter: every rank has packed its flat gradient (bf16 or fp32) into its symmetric staging buffer and the
//                  ranks have exchanged "ready" flags. Rank r then sums elements [start, start + per) of all ranks'
//                  buffers with 16-byte peer loads (8 elements per thread) in a fixed rank order (deterministic),
//                  scales by 1/world, writes its fp32 shard gradient and per-block sums of squares (for the global
//                  clip norm). This replaces reduce_scatter + the cast and scale kernels.
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

// 8 consecutive elements of a bf16 (dtype 1) or fp32 (dtype 0) buffer as floats: one 16-byte or two 16-byte loads
__device__ __forceinline__ void load8(const void* base, int64_t i, int dtype, float* out) {
  if (dtype == 0) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
    const float4 a = p[0], b = p[1];
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
    const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const bf16*>(base) + i);
    const bf16* v = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) out[k] = __bfloat162float(v[k]);
  }
}

__device__ __forceinline__ void store8(void* base, int64_t i, int dtype, const float* in) {
  if (dtype == 0) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + i);
    p[0] = make_float4(in[0], in[1], in[2], in[3]);
    p[1] = make_float4(in[4], in[5], in[6], in[7]);
  } else {
    uint4 w;
    w.x = pack_bf16(in[0], in[1]);
    w.y = pack_bf16(in[2], in[3]);
    w.z = pack_bf16(in[4], in[5]);
    w.w = pack_bf16(in[6], in[7]);
    *reinterpret_cast<uint4*>(static_cast<bf16*>(base) + i) = w;
  }
}

// each thread reduces 8 consecutive elements of the shard: per peer one 16-byte (bf16) or 32-byte (fp32) NVLink
// load, summed in fixed rank order
__global__ void __launch_bounds__(256) zero_rs_kernel(const void* const* __restrict__ peers, int world, int dtype,
                                                      int64_t start, int64_t per, float inv_world,
                                                      float* __restrict__ shard, double* __restrict__ partial) {
  float sq = 0.f;
  const int64_t vecs = per / 8;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < vecs;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < world; ++r) {
      float x[8];
      load8(peers[r], start + 8 * t, dtype, x);
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] += x[k];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s[k] *= inv_world;
      sq += s[k] * s[k];
    }
    float4* out = reinterpret_cast<float4*>(shard + 8 * t);
    out[0] = make_float4(s[0], s[1], s[2], s[3]);
    out[1] = make_float4(s[4], s[5], s[6], s[7]);
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

// AdamW on 8 consecutive shard elements per thread, then one 16-byte (bf16) or 32-byte (fp32) store of the new values
// into every rank's parameter buffer (the all-gather). Elements past `valid` (padding) are left at zero.
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
  const int64_t vecs = per / 8;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < vecs;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i0 = 8 * t;
    float pv[8], mv[8], vv[8], gv[8];
    load8(master, i0, 0, pv);
    load8(m, i0, 0, mv);
    load8(v, i0, 0, vv);
    load8(grad, i0, 0, gv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (start + i0 + k >= valid) {  // padding past the last parameter stays zero
        pv[k] = mv[k] = vv[k] = 0.f;
        continue;
      }
      const float g = gv[k] * coef;
      mv[k] = h.beta1 * mv[k] + (1.f - h.beta1) * g;
      vv[k] = h.beta2 * vv[k] + (1.f - h.beta2) * g * g;
      pv[k] = pv[k] * decay - step_size * mv[k] / (sqrtf(vv[k]) / h.bias_correction2_sqrt + h.eps);
    }
    store8(master, i0, 0, pv);
    store8(m, i0, 0, mv);
    store8(v, i0, 0, vv);
    for (int r = 0; r < world; ++r) store8(peers[r], start + i0, dtype, pv);  // NVLink stores: the all-gather
  }
}

}  // namespace

// shards are a multiple of 8 elements (the Python side pads them), one thread per 8 elements
int zero_rs_blocks(int64_t per) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(592, (per / 8 + 255) / 256)));
}

void zero_reduce_scatter(const void* const* peers, int world, int dtype, int64_t start, int64_t per, float* shard,
                         double* partial, cudaStream_t stream) {
  if (per == 0) return;
  if (per % 8 || start % 8) throw std::runtime_error("zero_reduce_scatter: shard start and size must be multiples of 8");
  zero_rs_kernel<<<zero_rs_blocks(per), 256, 0, stream>>>(peers, world, dtype, start, per, 1.f / world, shard,
                                                          partial);
  check_cuda(cudaGetLastError(), "zero_reduce_scatter");
}

void zero_adamw_gather(float* master, float* m, float* v, const float* grad, const float* clip, const AdamHyper& h,
                       void* const* peers, int world, int dtype, int64_t start, int64_t per, int64_t valid,
                       cudaStream_t stream) {
  if (per == 0) return;
  if (per % 8 || start % 8) throw std::runtime_error("zero_adamw_gather: shard start and size must be multiples of 8");
  zero_adamw_gather_kernel<<<zero_rs_blocks(per), 256, 0, stream>>>(master, m, v, grad, clip, h, peers, world, dtype,
                                                                    start, per, valid);
  check_cuda(cudaGetLastError(), "zero_adamw_gather");
}

}  // namespace qw
