// Host launchers for the tcgen05 GEMM (gemm_tcgen05.cuh): dense linear layers and the grouped MoE expert GEMMs.
// Raw-pointer API (no torch headers here); argument validation lives in bindings.cpp.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>

#include "gemm_tcgen05.cuh"
#include "launchers.h"

namespace qw {
namespace gemm {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr)
      throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

static void require(bool ok, const char* what) {
  if (!ok) throw std::runtime_error(std::string("qw gemm: ") + what);
}

// 2-D bf16 map over a row-major [outer, inner] region with row stride `ld` elements; box = [box_outer, box_inner].
static CUtensorMap make_map(const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner, int box_outer) {
  // the driver call needs a current context; threads that have not touched the runtime yet (the autograd engine's
  // device threads) get the primary context of the current device here
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(dev);
  require((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  require((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes (ld % 8 == 0)");
  require(box_inner * 2 == 128, "swizzle-128 boxes are 64 bf16 wide");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("qw gemm: cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) +
                             ", inner " + std::to_string(inner) + ", outer " + std::to_string(outer) + ", ld " +
                             std::to_string(ld) + ", box " + std::to_string(box_inner) + "x" +
                             std::to_string(box_outer) + ", base " +
                             std::to_string(reinterpret_cast<uintptr_t>(ptr) % 1024) + " mod 1024)");
  return map;
}

}  // namespace gemm

// 3-D bf16 map over [batches][rows][inner] with row stride `ld` and batch stride `batch_stride` elements; the box is
// 64 elements (128 B, swizzle-128) x box_rows x 1. Coordinates past `rows` read as zeros, so a tile never reaches
// into the next batch.
CUtensorMap make_bf16_map_3d(const void* ptr, int64_t inner, int64_t rows, int64_t batches, int64_t ld,
                             int64_t batch_stride, int box_rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(dev);
  gemm::require((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  gemm::require((ld * 2) % 16 == 0 && (batch_stride * 2) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batches)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(batch_stride * 2)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = gemm::encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
                                 elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("qw: cuTensorMapEncodeTiled (3-D) failed (code " + std::to_string(static_cast<int>(r)) +
                             ", inner " + std::to_string(inner) + ", rows " + std::to_string(rows) + ", ld " +
                             std::to_string(ld) + ")");
  return map;
}

namespace gemm {

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Whether bf16 outputs go through the staged (coalesced) epilogue, the default; QW_GEMM_STAGED_EPI=0 keeps the
// per-thread stores.
static bool staged_epilogue_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("QW_GEMM_STAGED_EPI");
    return !(e && std::string(e) == "0");
  }();
  return on;
}

// Maps of the TMA epilogue (output, residual, raw gate|up); unused ones stay zero.
struct OutMaps {
  CUtensorMap out{}, res{}, gu{};
};

// A [rows, cols] bf16 map with 32-row x 64-column boxes (128-byte swizzle) for the TMA epilogue, or false when the
// buffer's alignment rules one out.
static bool epi_map(CUtensorMap& m, const void* ptr, int64_t cols, int64_t rows, int64_t ld) {
  if (!ptr || rows <= 0 || (reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16) return false;
  m = make_map(ptr, cols, rows, ld, 64, 32);
  return true;
}

// The staged epilogue moves 16-byte chunks: the buffer and its row stride (ld elements of esize bytes) must be
// 16-byte aligned.
static bool aligned16(const void* ptr, int64_t ld, int esize = 2) {
  return ptr && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (ld * esize) % 16 == 0;
}

template <int BN, int MODE, int EPI, bool A_MN, bool B_MN>
static void launch(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, int64_t total_tiles_bound,
                   cudaStream_t stream, const OutMaps& outs = OutMaps{}) {
  auto kernel = gemm_kernel<BN, MODE, EPI, A_MN, B_MN>;
  static bool configured = false;
  const int smem = Smem<BN>::kTotal;
  if (!configured) {
    check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "smem attribute");
    configured = true;
  }
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms(), total_tiles_bound)));
  kernel<<<grid, kThreads, smem, stream>>>(ma, mb, outs.out, outs.res, outs.gu, p);
  check_cuda(cudaGetLastError(), "gemm launch");
}

static Params base_params() {
  Params p{};
  p.alpha = 1.f;
  return p;
}

}  // namespace gemm

using namespace gemm;

// ------------------------------------------------------------------------------------------------ dense
// out[M,N] = x[M,K] @ w[N,K]^T (+bias[N]) (+residual[M,N])
void linear_fwd(const bf16* x, int64_t ldx, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                const float* bias, const bf16* residual, int64_t ldr, void* out, int64_t ldo, bool out_fp32,
                cudaStream_t stream) {
  if (M == 0 || N == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.M = M; p.N = N; p.K = K;
  p.num_groups = 1;
  p.n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.max_tiles = INT_MAX;
  p.out = out; p.ldo = ldo; p.out_fp32 = out_fp32;
  p.bias = bias;
  p.residual = residual; p.ldr = ldr;
  auto ma = make_map(x, K, M, ldx, 64, kBM);
  auto mb = make_map(w, K, N, ldw, 64, BN);
  OutMaps outs;
  p.tma_out = staged_epilogue_enabled() && !out_fp32 && epi_map(outs.out, out, N, M, ldo) &&
              (!residual || epi_map(outs.res, residual, N, M, ldr));
  p.staged_out = !p.tma_out && staged_epilogue_enabled() && N % 8 == 0 && aligned16(out, ldo, out_fp32 ? 4 : 2) &&
                 (!residual || (!out_fp32 && aligned16(residual, ldr)));
  launch<BN, kGroupM, kEpiStore, false, false>(ma, mb, p, ((M + kBM - 1) / kBM) * p.n_tiles, stream, outs);
}

// dx[M,K] (+)= dy[M,N] @ w[N,K]
void linear_dgrad(const bf16* dy, int64_t lddy, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K, void* dx,
                  int64_t lddx, bool out_fp32, bool accumulate, cudaStream_t stream) {
  if (M == 0 || K == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.M = M; p.N = K; p.K = N;
  p.num_groups = 1;
  p.n_tiles = static_cast<int>((K + BN - 1) / BN);
  p.max_tiles = INT_MAX;
  p.out = dx; p.ldo = lddx; p.out_fp32 = out_fp32; p.accumulate = accumulate;
  auto ma = make_map(dy, N, M, lddy, 64, kBM);
  auto mb = make_map(w, K, N, ldw, 64, 64);
  OutMaps outs;
  p.tma_out = staged_epilogue_enabled() && !out_fp32 && !accumulate && epi_map(outs.out, dx, K, M, lddx);
  p.staged_out = !p.tma_out && staged_epilogue_enabled() && (out_fp32 || !accumulate) && K % 8 == 0 &&
                 aligned16(dx, lddx, out_fp32 ? 4 : 2);
  launch<BN, kGroupM, kEpiStore, false, true>(ma, mb, p, ((M + kBM - 1) / kBM) * p.n_tiles, stream, outs);
}

// dw[N,K] (+)= dy[T,N]^T @ x[T,K]
void linear_wgrad(const bf16* dy, int64_t lddy, const bf16* x, int64_t ldx, int64_t T, int64_t N, int64_t K, void* dw,
                  int64_t lddw, bool out_fp32, bool accumulate, cudaStream_t stream) {
  if (N == 0 || K == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.M = N; p.N = K; p.K = T;
  p.num_groups = 1;
  p.m_tiles = static_cast<int>((N + kBM - 1) / kBM);
  p.n_tiles = static_cast<int>((K + BN - 1) / BN);
  p.out = dw; p.ldo = lddw; p.out_fp32 = out_fp32; p.accumulate = accumulate;
  p.staged_out = staged_epilogue_enabled() && (out_fp32 || !accumulate) && K % 8 == 0 &&
                 aligned16(dw, lddw, out_fp32 ? 4 : 2);
  auto ma = make_map(dy, N, std::max<int64_t>(T, 1), lddy, 64, 64);
  auto mb = make_map(x, K, std::max<int64_t>(T, 1), ldx, 64, 64);
  launch<BN, kGroupK, kEpiStore, true, true>(ma, mb, p, static_cast<int64_t>(p.m_tiles) * p.n_tiles, stream);
}

// Tensor-parallel partial products written straight into the owners' staging buffers (peer stores over NVLink):
// row m of the [M, N] result goes to rank m / peer_rows, slot `peer_slot`. bf16, no bias (the reduction adds it).
void linear_fwd_peer(const bf16* x, int64_t ldx, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                     void* const* peer_out, int64_t peer_rows, int peer_slot, cudaStream_t stream) {
  if (M == 0 || N == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.M = M; p.N = N; p.K = K;
  p.num_groups = 1;
  p.n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.max_tiles = INT_MAX;
  p.out = nullptr; p.ldo = N; p.out_fp32 = 0;
  p.peer_out = peer_out; p.peer_rows = peer_rows; p.peer_slot = peer_slot;
  auto ma = make_map(x, K, M, ldx, 64, kBM);
  auto mb = make_map(w, K, N, ldw, 64, BN);
  launch<BN, kGroupM, kEpiStore, false, false>(ma, mb, p, ((M + kBM - 1) / kBM) * p.n_tiles, stream);
}

// dx partial [M, K] = dy[M, N] @ w[N, K] into the owners' staging buffers (see linear_fwd_peer)
void linear_dgrad_peer(const bf16* dy, int64_t lddy, const bf16* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                       void* const* peer_out, int64_t peer_rows, int peer_slot, cudaStream_t stream) {
  if (M == 0 || K == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.M = M; p.N = K; p.K = N;
  p.num_groups = 1;
  p.n_tiles = static_cast<int>((K + BN - 1) / BN);
  p.max_tiles = INT_MAX;
  p.out = nullptr; p.ldo = K; p.out_fp32 = 0;
  p.peer_out = peer_out; p.peer_rows = peer_rows; p.peer_slot = peer_slot;
  auto ma = make_map(dy, N, M, lddy, 64, kBM);
  auto mb = make_map(w, K, N, ldw, 64, 64);
  launch<BN, kGroupM, kEpiStore, false, true>(ma, mb, p, ((M + kBM - 1) / kBM) * p.n_tiles, stream);
}

// partial[c][N,K] = dy[rows of chunk c, N]^T @ x[rows of chunk c, K] for chunks of `chunk` rows (a multiple of 64):
// split-K for weight gradients whose output is too small to fill the GPU (the caller reduces the partials)
void linear_wgrad_chunks(const bf16* dy, int64_t lddy, const bf16* x, int64_t ldx, int64_t T, int64_t N, int64_t K,
                         int64_t chunk, float* partial, cudaStream_t stream) {
  if (N == 0 || K == 0 || T == 0) return;
  require(chunk % kBK == 0, "split-K chunk must be a multiple of 64 rows");
  constexpr int BN = 256;
  Params p = base_params();
  p.M = N; p.N = K; p.K = T;
  p.num_groups = static_cast<int>((T + chunk - 1) / chunk);
  p.k_chunk = static_cast<int>(chunk);
  p.m_tiles = static_cast<int>((N + kBM - 1) / kBM);
  p.n_tiles = static_cast<int>((K + BN - 1) / BN);
  p.out = partial; p.ldo = K; p.out_fp32 = 1;
  p.out_group_stride = N * K;
  p.staged_out = staged_epilogue_enabled() && K % 8 == 0 && aligned16(partial, K, 4);
  auto ma = make_map(dy, N, T, lddy, 64, 64);
  auto mb = make_map(x, K, T, ldx, 64, 64);
  launch<BN, kGroupK, kEpiStore, true, true>(ma, mb, p,
                                             static_cast<int64_t>(p.m_tiles) * p.n_tiles * p.num_groups, stream);
}

// ------------------------------------------------------------------------------------------------ grouped (MoE)
// Expert e owns rows [offsets[e], offsets[e] + counts[e]) of the permuted activations; offsets are multiples of
// 128 and rows [counts[e], roundup128(counts[e])) are zero padding (written as zeros by every producer).

// h[R,F] = silu(x Wg^T) * (x Wu^T) ; optional raw gu[R,2F]    (w_gate_up [E, 2F, H])
void moe_gate_up_fwd(const bf16* x, const bf16* w_gate_up, const int* counts, const int* offsets, int64_t R, int64_t G,
                     int64_t E, int64_t H, int64_t F, bf16* h, bf16* gu, cudaStream_t stream) {
  if (R == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.N = 2 * F; p.K = H;
  p.num_groups = static_cast<int>(G);
  p.expert_mod = static_cast<int>(E);
  p.group_rows = counts; p.group_off = offsets;
  p.b_group_rows = static_cast<int>(2 * F);
  p.dual_b_offset = static_cast<int>(F);
  p.ffn = static_cast<int>(F);
  p.n_tiles = static_cast<int>((F + BN / 2 - 1) / (BN / 2));
  p.max_tiles = static_cast<int>(((R + kBM - 1) / kBM) * p.n_tiles);
  p.out = h; p.ldo = F;
  p.zero_pad_rows = 1;
  p.gu_out = gu;
  auto ma = make_map(x, H, R, H, 64, kBM);
  auto mb = make_map(w_gate_up, H, E * 2 * F, H, 64, BN / 2);
  OutMaps outs;
  p.tma_out = staged_epilogue_enabled() && F % 8 == 0 && epi_map(outs.out, h, F, R, F) &&
              (!gu || epi_map(outs.gu, gu, 2 * F, R, 2 * F));
  p.staged_out = !p.tma_out && staged_epilogue_enabled() && F % 64 == 0 && aligned16(h, F) &&
                 (!gu || aligned16(gu, 2 * F));
  launch<BN, kGroupM, kEpiSwiGLU, false, false>(ma, mb, p, p.max_tiles, stream, outs);
}

// y[R,H] = h[R,F] @ w_down[e]^T   (w_down [E, H, F]). With `peer_out`, row r is stored over NVLink into rank
// r / peer_rows's buffer at row peer_slot * peer_rows + r % peer_rows instead (the expert-parallel combine push:
// rows are laid out [source rank][local expert][slot], so peer_rows = local * slot and peer_slot = this rank);
// padding rows are not written then.
void moe_down_fwd(const bf16* h, const bf16* w_down, const int* counts, const int* offsets, int64_t R, int64_t G,
                  int64_t E, int64_t H, int64_t F, bf16* y, cudaStream_t stream, void* const* peer_out,
                  int64_t peer_rows, int peer_slot) {
  if (R == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.N = H; p.K = F;
  p.num_groups = static_cast<int>(G);
  p.expert_mod = static_cast<int>(E);
  p.group_rows = counts; p.group_off = offsets;
  p.b_group_rows = static_cast<int>(H);
  p.n_tiles = static_cast<int>((H + BN - 1) / BN);
  p.max_tiles = static_cast<int>(((R + kBM - 1) / kBM) * p.n_tiles);
  p.out = y; p.ldo = H;
  p.zero_pad_rows = peer_out ? 0 : 1;
  p.peer_out = peer_out; p.peer_rows = peer_rows; p.peer_slot = peer_slot;
  auto ma = make_map(h, F, R, F, 64, kBM);
  auto mb = make_map(w_down, F, E * H, F, 64, BN);
  OutMaps outs;
  p.tma_out = staged_epilogue_enabled() && !peer_out && epi_map(outs.out, y, H, R, H);
  launch<BN, kGroupM, kEpiStore, false, false>(ma, mb, p, p.max_tiles, stream, outs);
}

// a = dy @ w_down[e] ; dgu = [w*a*u*silu'(g) | w*a*silu(g)] ; h_w = w*silu(g)*u ; dw_partial[r,t] = <a,h> per tile
void moe_down_bwd(const bf16* dy, const bf16* w_down, const int* counts, const int* offsets, int64_t R, int64_t G,
                  int64_t E, int64_t H, int64_t F, const bf16* gu, const float* route_w, bf16* dgu, bf16* h_weighted,
                  float* dw_partial, int dw_tiles, cudaStream_t stream) {
  if (R == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.N = F; p.K = H;
  p.num_groups = static_cast<int>(G);
  p.expert_mod = static_cast<int>(E);
  p.group_rows = counts; p.group_off = offsets;
  p.b_group_rows = static_cast<int>(H);
  p.ffn = static_cast<int>(F);
  p.n_tiles = static_cast<int>((F + BN - 1) / BN);
  require(p.n_tiles == dw_tiles, "dw_partial tile count mismatch");
  p.max_tiles = static_cast<int>(((R + kBM - 1) / kBM) * p.n_tiles);
  p.out = dgu;
  p.gu_in = gu;
  p.route_w = route_w;
  p.h_out = h_weighted;
  p.dw_partial = dw_partial;
  p.zero_pad_rows = 1;
  auto ma = make_map(dy, H, R, H, 64, kBM);
  auto mb = make_map(w_down, F, E * H, F, 64, 64);
  launch<BN, kGroupM, kEpiSwiGLUBwd, false, true>(ma, mb, p, p.max_tiles, stream);
}

int moe_dw_tiles(int64_t F) { return static_cast<int>((F + 255) / 256); }

// dx[R,H] = dgu[R,2F] @ w_gate_up[e]; `peer_out` as in moe_down_fwd (the expert-parallel input-gradient push)
void moe_gate_up_dgrad(const bf16* dgu, const bf16* w_gate_up, const int* counts, const int* offsets, int64_t R,
                       int64_t G, int64_t E, int64_t H, int64_t F, bf16* dx, cudaStream_t stream,
                       void* const* peer_out, int64_t peer_rows, int peer_slot) {
  if (R == 0) return;
  constexpr int BN = 256;
  Params p = base_params();
  p.N = H; p.K = 2 * F;
  p.num_groups = static_cast<int>(G);
  p.expert_mod = static_cast<int>(E);
  p.group_rows = counts; p.group_off = offsets;
  p.b_group_rows = static_cast<int>(2 * F);
  p.n_tiles = static_cast<int>((H + BN - 1) / BN);
  p.max_tiles = static_cast<int>(((R + kBM - 1) / kBM) * p.n_tiles);
  p.out = dx; p.ldo = H;
  p.zero_pad_rows = peer_out ? 0 : 1;
  p.peer_out = peer_out; p.peer_rows = peer_rows; p.peer_slot = peer_slot;
  auto ma = make_map(dgu, 2 * F, R, 2 * F, 64, kBM);
  auto mb = make_map(w_gate_up, H, E * 2 * F, H, 64, 64);
  OutMaps outs;
  p.tma_out = staged_epilogue_enabled() && !peer_out && epi_map(outs.out, dx, H, R, H);
  launch<BN, kGroupM, kEpiStore, false, true>(ma, mb, p, p.max_tiles, stream, outs);
}

// out[e][M,N] (+)= a[rows_e, M]^T @ b[rows_e, N]
void moe_wgrad(const bf16* a, const bf16* b, const int* counts, const int* offsets, int64_t R, int64_t E, int segments,
               int64_t M, int64_t N, void* out, bool out_fp32, bool accumulate, float alpha, cudaStream_t stream) {
  constexpr int BN = 256;
  Params p = base_params();
  p.M = M; p.N = N;
  p.num_groups = static_cast<int>(E);
  p.k_segments = segments;
  p.alpha = alpha;
  p.group_rows = counts; p.group_off = offsets;
  p.m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  p.n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.out = out; p.ldo = N;
  p.out_group_stride = M * N;
  p.out_fp32 = out_fp32; p.accumulate = accumulate;
  p.staged_out = staged_epilogue_enabled() && (out_fp32 || !accumulate) && N % 8 == 0 &&
                 aligned16(out, N, out_fp32 ? 4 : 2);
  auto ma = make_map(a, M, std::max<int64_t>(R, 1), M, 64, 64);
  auto mb = make_map(b, N, std::max<int64_t>(R, 1), N, 64, 64);
  launch<BN, kGroupK, kEpiStore, true, true>(ma, mb, p, static_cast<int64_t>(p.m_tiles) * p.n_tiles * E, stream);
}

namespace {
// out[r, c] (+)= sum over chunks (fixed order) of partial[chunk][r][c]: the tail of a split-K weight gradient
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ partial, int chunks, int rows,
                                                            int cols, void* __restrict__ out, int64_t ldo,
                                                            int out_fp32, int accumulate) {
  const int64_t total = static_cast<int64_t>(rows) * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int c = 0; c < chunks; ++c) acc += partial[c * total + i];
    const int64_t at = (i / cols) * ldo + i % cols;
    if (out_fp32) {
      float* o = static_cast<float*>(out) + at;
      *o = accumulate ? *o + acc : acc;
    } else {
      bf16* o = static_cast<bf16*>(out) + at;
      *o = __float2bfloat16(accumulate ? __bfloat162float(*o) + acc : acc);
    }
  }
}
}  // namespace

// Split-K factor for a dense weight gradient whose output tiles cannot fill the GPU (1 = no split): enough row
// chunks for about two waves of output tiles, each chunk at least 1024 rows.
int wgrad_split(int64_t T, int64_t N, int64_t K) {
  const int64_t tiles = ((N + kBM - 1) / kBM) * ((K + 255) / 256);
  if (tiles >= num_sms() || T < 4096) return 1;
  const int64_t want = (2 * num_sms() + tiles - 1) / tiles;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, T / 1024)));
}

void splitk_reduce(const float* partial, int chunks, int64_t rows, int64_t cols, void* out, int64_t ldo,
                   bool out_fp32, bool accumulate, cudaStream_t stream) {
  const int64_t total = rows * cols;
  if (total == 0) return;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(4 * num_sms(), (total + 255) / 256)));
  splitk_reduce_kernel<<<grid, 256, 0, stream>>>(partial, chunks, static_cast<int>(rows), static_cast<int>(cols), out,
                                                 ldo, out_fp32 ? 1 : 0, accumulate ? 1 : 0);
  check_cuda(cudaGetLastError(), "splitk_reduce");
}

int gemm_status(bool clear) { return read_status_word(clear); }

// Arms (buf != null: kTraceTiles x 8 int64 slots) or disarms the per-tile timestamps of CTA 0 of every GEMM launch.
void gemm_trace(void* buf) {
  unsigned long long* ptr = static_cast<unsigned long long*>(buf);
  check_cuda(cudaMemcpyToSymbol(g_gemm_trace, &ptr, sizeof(ptr)), "gemm trace");
}

}  // namespace qw
