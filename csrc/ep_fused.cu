// Fused expert-parallel exchange over NVLink peer memory (symmetric buffers mapped into every rank).
//
//  dispatch: one warp per route reads its token row and stores it, with its routing weight, straight into the
//            owning rank's receive buffer at row (source * local + local_expert) * slot + position (the layout the
//            grouped expert GEMMs read); block 0 also stores this rank's per-expert kept counts there. This replaces
//            the local permute, its send buffer and three all-to-all exchanges. The last block to finish publishes
//            `epoch` into every peer's flag[me] with a system-scope release store.
//  pad fix:  after the flag wait, the receiver zeroes each segment's rows [count, round_up(count, 128)) so the
//            128-row GEMM tiles read zeros (and zero weights) past the last routed row.
//  signal:   after the expert GEMM's peer-store epilogue (gemm_tcgen05.cuh) pushed every output row into its source
//            rank's return buffer, release flags to every peer; each source then reduces its top-k rows locally
//            (combine_kernel / combine_grad_kernel in moe_routing.cu) once every expert rank has signalled.
// Only plain loads and stores to peer memory are used (no multimem, no TMA). Flag waits are p2p_wait (bounded).
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

__device__ __forceinline__ void st_release_sys(int* addr, int value) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(addr), "r"(value) : "memory");
}

struct DispatchArgs {
  const bf16* x;         // [T, H] rows to send
  int64_t T;
  int k, H;
  const int* route_row;  // [T*k] sender-layout row e * slot + pos, or -1 (dropped)
  const float* top_w;    // [T*k] or nullptr
  const int* kept;       // [E] or nullptr
  int E, local, slot, me, world;
  uint8_t* const* peer;  // [world] receive buffer base of every rank
  int64_t w_off, c_off;  // byte offsets of the weight and count regions in the buffer
  int* const* peer_flags;
  int epoch;
  unsigned int* done;
};

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const DispatchArgs a) {
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t routes = a.T * a.k;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * warps + warp; r < routes;
       r += static_cast<int64_t>(gridDim.x) * warps) {
    const int row = a.route_row[r];
    if (row < 0) continue;
    const int e = row / a.slot, pos = row % a.slot;
    if (!in_bounds(e, a.E)) continue;  // QW_DEBUG_BOUNDS: a route past the last expert would write outside a peer
    const int d = e / a.local, le = e % a.local;
    const int64_t rrow = static_cast<int64_t>(a.me * a.local + le) * a.slot + pos;
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (r / a.k) * a.H);
    uint4* dst = reinterpret_cast<uint4*>(a.peer[d] + rrow * a.H * 2);
    for (int c = lane; c < a.H / 8; c += 32) dst[c] = src[c];
    if (a.top_w && lane == 0) reinterpret_cast<float*>(a.peer[d] + a.w_off)[rrow] = a.top_w[r];
  }
  if (a.kept && blockIdx.x == 0) {
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
      const int d = e / a.local, le = e % a.local;
      reinterpret_cast<int*>(a.peer[d] + a.c_off)[a.me * a.local + le] = a.kept[e];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x - 1) {  // every block's stores are fenced: publish to all peers
      __threadfence_system();
      for (int d = 0; d < a.world; ++d) st_release_sys(a.peer_flags[d] + a.me, a.epoch);
      *a.done = 0;
    }
  }
}

// zero rows [count, round_up(count, 128)) of every segment g (and their weights); block per segment
__global__ void ep_pad_kernel(const int* __restrict__ counts, int slot, int H, bf16* __restrict__ rows,
                              float* __restrict__ w) {
  const int g = blockIdx.x;
  const int n = counts[g];
  const int end = min(slot, (n + 127) / 128 * 128);
  const int64_t base = static_cast<int64_t>(g) * slot;
  for (int r = n + threadIdx.y; r < end; r += blockDim.y) {
    uint4* dst = reinterpret_cast<uint4*>(rows + (base + r) * H);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    if (w && threadIdx.x == 0) w[base + r] = 0.f;
  }
}

__global__ void ep_signal_kernel(int* const* __restrict__ peer_flags, int world, int me, int epoch) {
  __threadfence_system();
  __syncthreads();
  const int d = threadIdx.x;
  if (d < world) st_release_sys(peer_flags[d] + me, epoch);
}

}  // namespace

void ep_dispatch(const bf16* x, int64_t T, int k, int H, const int* route_row, const float* top_w, const int* kept,
                 int E, int local, int slot, int me, int world, uint8_t* const* peer, int64_t w_off, int64_t c_off,
                 int* const* peer_flags, int epoch, unsigned int* done, cudaStream_t stream) {
  if (H % 8) throw std::runtime_error("ep_dispatch: hidden size must be a multiple of 8");
  if (k > 8) throw std::runtime_error("ep_dispatch: top-k above 8");
  DispatchArgs a{x, T, k, H, route_row, top_w, kept, E, local, slot, me, world, peer, w_off, c_off, peer_flags, epoch,
                 done};
  const int64_t routes = T * k;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(4 * 148, (routes + 7) / 8)));
  ep_dispatch_kernel<<<blocks, 256, 0, stream>>>(a);
  check_cuda(cudaGetLastError(), "ep_dispatch");
}

void ep_pad(const int* counts, int groups, int slot, int H, bf16* rows, float* w, cudaStream_t stream) {
  if (groups == 0) return;
  ep_pad_kernel<<<groups, dim3(32, 8), 0, stream>>>(counts, slot, H, rows, w);
  check_cuda(cudaGetLastError(), "ep_pad");
}

void ep_signal(int* const* peer_flags, int world, int me, int epoch, cudaStream_t stream) {
  ep_signal_kernel<<<1, 32, 0, stream>>>(peer_flags, world, me, epoch);
  check_cuda(cudaGetLastError(), "ep_signal");
}

int ep_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
