// Expert-parallel decode over NVLink peer memory.
//
// Every rank of the expert group decodes the same tokens (SPMD: the embeddings, attention and router are replicated);
// at each MoE layer a rank runs only the experts it holds, and the per-token partial outputs are exchanged by peer
// stores instead of an all-reduce:
//
//   ep_decode_tick   the decode step counter += 1 (the first kernel of every step, so a CUDA graph replays with a
//                    fresh target without re-capturing)
//   ep_decode_push   one block per token: partial[t] = sum over its k routes of top_w * y[slot] in fp32 (the rows of
//                    routes to other ranks' experts were zeroed, so they add nothing), stored into slot `me` of every
//                    rank's exchange plane [world][Tmax][H] with 16-byte NVLink stores; the last block releases
//                    target = step * layers + layer + 1 into every peer's flag[me] (system scope)
//   ep_decode_wait   one thread per peer: bounded acquire-spin until that peer's flag reached the target
//
// The sum of the partials (fixed rank order, so every rank computes bit-identical activations) is fused into the next
// layer's norm (decode.cu combine_norm_kernel). Flags only grow (step * layers + layer + 1), so one flag word per
// peer serves every layer. The exchange buffer has two planes per layer, alternating with the step's parity
// (plane = (step & 1) * layers + layer): a rank cannot start step n+2 before every peer has pushed step n+1, which
// each does only after it read its step-n planes, so no plane is overwritten while a peer still reads it.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

__device__ __forceinline__ void st_release_sys(int* addr, int value) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(addr), "r"(value) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__global__ void ep_decode_tick_kernel(int* step) { *step += 1; }

__global__ void __launch_bounds__(256) ep_decode_push_kernel(const bf16* __restrict__ y, const int* __restrict__ slot,
                                                             const float* __restrict__ top_w, int k, int T, int H,
                                                             int tstride, float* const* __restrict__ peers,
                                                             int64_t plane_floats,
                                                             int layer, int layers, int me, int world,
                                                             int* const* __restrict__ peer_flags,
                                                             const int* __restrict__ step,
                                                             unsigned int* __restrict__ done) {
  const int t = blockIdx.x;
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const float w = top_w[t * k + j];
      const uint2 raw = *reinterpret_cast<const uint2*>(y + static_cast<int64_t>(slot[t * k + j]) * H + h);
      const bf16* v = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += w * __bfloat162float(v[i]);
    }
    const float4 out = make_float4(acc[0], acc[1], acc[2], acc[3]);
    const int plane = (*step & 1) * layers + layer;
    const int64_t at = plane * plane_floats + (static_cast<int64_t>(me) * tstride + t) * H + h;
    for (int d = 0; d < world; ++d) *reinterpret_cast<float4*>(peers[d] + at) = out;  // NVLink stores
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {  // every block's stores are fenced: publish to all peers
      __threadfence_system();
      const int target = *step * layers + layer + 1;
      for (int d = 0; d < world; ++d) st_release_sys(peer_flags[d] + me, target);
      *done = 0;
    }
  }
}

__global__ void ep_decode_wait_kernel(const int* __restrict__ flags, int world, const int* __restrict__ step,
                                      int layer, int layers, uint64_t timeout_ns) {
  const int s = threadIdx.x;
  if (s >= world) return;
  const int target = *step * layers + layer + 1;
  if (ld_acquire_sys(flags + s) >= target) return;
  const uint64_t start = globaltimer();
  while (ld_acquire_sys(flags + s) < target) {
    if (globaltimer() - start > timeout_ns) {
      set_status(kTimeoutPeer);
      return;
    }
  }
}

}  // namespace

void ep_decode_tick(int* step, cudaStream_t stream) {
  ep_decode_tick_kernel<<<1, 1, 0, stream>>>(step);
  check_cuda(cudaGetLastError(), "ep_decode_tick");
}

void ep_decode_push(const bf16* y, const int* slot, const float* top_w, int k, int T, int H, int tstride,
                    float* const* peers, int64_t plane_floats, int layer, int layers, int me, int world,
                    int* const* peer_flags, const int* step, unsigned int* done, cudaStream_t stream) {
  if (T == 0) return;
  if (H % 4) throw std::runtime_error("ep_decode_push: hidden size must be a multiple of 4");
  ep_decode_push_kernel<<<T, 256, 0, stream>>>(y, slot, top_w, k, T, H, tstride, peers, plane_floats, layer, layers,
                                               me, world, peer_flags, step, done);
  check_cuda(cudaGetLastError(), "ep_decode_push");
}

void ep_decode_wait(const int* flags, int world, const int* step, int layer, int layers, double timeout_s,
                    cudaStream_t stream) {
  ep_decode_wait_kernel<<<1, 32, 0, stream>>>(flags, world, step, layer, layers,
                                              static_cast<uint64_t>(timeout_s * 1e9));
  check_cuda(cudaGetLastError(), "ep_decode_wait");
}

int ep_decode_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
