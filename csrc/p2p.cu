// Peer-to-peer exchange over NVLink: SM-issued stores into peers' symmetric buffers plus release/acquire flags.
//
// push:  block (chunk c, destination d) copies its slice of my block d (or, broadcasting, of my one block) into peer
//        d's receive buffer at slot `me`;
//        every block fences (system scope) and bumps a local counter; the last block for d publishes
//        `epoch` into peer d's flag[me] with a system-scope release store.
// wait:  one thread per source spins on my flag[source] with acquire loads, bounded by a %globaltimer budget;
//        on timeout it records kTimeoutPeer in the status word and returns (no trap, no endless loop).
//
// Only plain loads/stores to peer memory are used (no multimem, no TMA from peer memory).
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

// src_stride 1: block d of src goes to peer d (all-to-all); 0: the one block src goes to every peer (all-gather)
__global__ void p2p_push_kernel(const uint4* __restrict__ src, int64_t blk_vecs, int src_stride,
                                uint4* const* __restrict__ peer_bufs, int* const* __restrict__ peer_flags, int me,
                                int epoch, unsigned int* __restrict__ done) {
  const int d = blockIdx.y;
  const int chunks = gridDim.x;
  const int64_t per = (blk_vecs + chunks - 1) / chunks;
  const int64_t lo = blockIdx.x * per;
  const int64_t hi = min(blk_vecs, lo + per);
  const uint4* s = src + static_cast<int64_t>(d) * src_stride * blk_vecs;
  uint4* dst = peer_bufs[d] + static_cast<int64_t>(me) * blk_vecs;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = s[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(&done[d], 1u);
    if (prev == static_cast<unsigned>(chunks - 1)) {
      __threadfence_system();
      st_release_sys(peer_flags[d] + me, epoch);
      done[d] = 0;
    }
  }
}

__global__ void p2p_wait_kernel(const int* __restrict__ flags, int world, int epoch, uint64_t timeout_ns) {
  const int s = threadIdx.x;
  if (s >= world) return;
  if (ld_acquire_sys(flags + s) >= epoch) return;
  const uint64_t start = globaltimer();
  while (ld_acquire_sys(flags + s) < epoch) {
    if (globaltimer() - start > timeout_ns) {
      set_status(kTimeoutPeer);
      return;
    }
  }
}

}  // namespace

void p2p_push(const void* src, int64_t block_bytes, void* const* peer_bufs, int* const* peer_flags, int world, int me,
              int epoch, unsigned int* done, cudaStream_t stream) {
  if (block_bytes % 16) throw std::runtime_error("p2p_push: block bytes must be a multiple of 16");
  const int64_t vecs = block_bytes / 16;
  const int chunks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(132, (vecs + 4095) / 4096)));
  dim3 grid(chunks, world);
  p2p_push_kernel<<<grid, 512, 0, stream>>>(static_cast<const uint4*>(src), vecs, 1,
                                            reinterpret_cast<uint4* const*>(peer_bufs), peer_flags, me, epoch, done);
  check_cuda(cudaGetLastError(), "p2p_push");
}

void p2p_broadcast(const void* src, int64_t block_bytes, void* const* peer_bufs, int* const* peer_flags, int world,
                   int me, int epoch, unsigned int* done, cudaStream_t stream) {
  if (block_bytes % 16) throw std::runtime_error("p2p_broadcast: block bytes must be a multiple of 16");
  const int64_t vecs = block_bytes / 16;
  const int chunks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(132, (vecs + 4095) / 4096)));
  dim3 grid(chunks, world);
  p2p_push_kernel<<<grid, 512, 0, stream>>>(static_cast<const uint4*>(src), vecs, 0,
                                            reinterpret_cast<uint4* const*>(peer_bufs), peer_flags, me, epoch, done);
  check_cuda(cudaGetLastError(), "p2p_broadcast");
}

void p2p_wait(const int* flags, int world, int epoch, double timeout_s, cudaStream_t stream) {
  p2p_wait_kernel<<<1, 32, 0, stream>>>(flags, world, epoch, static_cast<uint64_t>(timeout_s * 1e9));
  check_cuda(cudaGetLastError(), "p2p_wait");
}

int p2p_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
