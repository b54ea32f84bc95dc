// Allocation-free RMSNorm backward: a C entry point for callers that are not allowed to allocate device memory.
//
// This entry point has no counterpart in the reference implementation; it exists for integrators.
//
// Who needs it: host applications that own the whole device-memory budget and hand kernels only pre-placed
// buffers (serving runtimes that reserve memory up front, plugin hosts that forbid allocation after start-up),
// and code paths that must not call cudaMalloc/cudaFree because those calls can synchronise the device. Such a
// caller still passes every input and output buffer; the only extra memory this routine needs, the per-block
// partial sums of the weight gradient, lives in a file-scope device array of fixed size that every GPU loading
// this library holds until the process exits.
//
// Contract:
//   * dy, x: bf16 [rows, hidden] row-major; weight: fp32 [hidden]; rstd: fp32 [rows] (1/sqrt(mean(x^2)+eps) from
//     the forward pass); dx: bf16 [rows, hidden] (written); dweight: fp32 [hidden] (overwritten, not accumulated).
//   * hidden must be a multiple of 8, and dy, x and dx must start on a 16-byte boundary (rows are read and written
//     as 16-byte vectors); weight, rstd and dweight must be 4-byte aligned. Anything else is rejected with
//     QW_NOALLOC_BAD_ARGUMENT before anything runs, so a view at an odd element offset gets an error code, not a
//     misaligned-address fault.
//   * ceil(rows / 256) * hidden must not exceed QW_NOALLOC_SCRATCH_FLOATS (4,194,304 floats = 16 MiB); larger
//     problems are rejected with QW_NOALLOC_TOO_LARGE before anything runs.
//   * rows == 0 is valid: nothing is read and dweight is set to zero.
//   * A CUDA error already pending on the calling thread (from earlier, unrelated work) is left in place and the
//     call returns QW_NOALLOC_PENDING_ERROR without launching, so it never reports or clears an error it did not
//     cause; QW_NOALLOC_CUDA_ERROR means that this call's own set-up or launch failed.
//   * The first call on a device looks up the device address of the scratch array for that device
//     (cudaGetSymbolAddress, with that device current); make that first call before any stream capture.
//   * Every call shares the one scratch array, which keeps the last call's partial sums. Calls that can overlap on
//     the GPU (different streams without ordering between them) race on it and must not be issued that way.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "noalloc.h"

namespace {

constexpr int kRowsPerBlock = 256;
constexpr int kWarps = 8;

static __device__ __align__(256) float qw_noalloc_scratch[QW_NOALLOC_SCRATCH_FLOATS];

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// dx = rstd * (w*dy - xhat * mean(w*dy*xhat)); this block's column partials of dy*xhat go to scratch[block, :].
// Dynamic shared memory: kWarps * hidden floats (one partial row per warp).
__global__ void rms_bwd_partials(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                 const float* __restrict__ w, const float* __restrict__ rstd,
                                 __nv_bfloat16* __restrict__ dx, float* __restrict__ scratch, int64_t rows,
                                 int hidden) {
  extern __shared__ float part[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* mine = part + warp * hidden;
  for (int c = lane; c < hidden; c += 32) mine[c] = 0.f;
  __syncwarp();
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock;
  const int64_t last = first + kRowsPerBlock < rows ? first + kRowsPerBlock : rows;
  for (int64_t row = first + warp; row < last; row += kWarps) {
    const float r = rstd[row];
    float s = 0.f;
    for (int c = lane * 8; c < hidden; c += 256) {
      const uint4 dr = *reinterpret_cast<const uint4*>(dy + row * hidden + c);
      const uint4 xr = *reinterpret_cast<const uint4*>(x + row * hidden + c);
      const __nv_bfloat16* dv = reinterpret_cast<const __nv_bfloat16*>(&dr);
      const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&xr);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += __bfloat162float(dv[j]) * w[c + j] * (__bfloat162float(xv[j]) * r);
    }
    s = warp_sum(s) / hidden;
    for (int c = lane * 8; c < hidden; c += 256) {
      const uint4 dr = *reinterpret_cast<const uint4*>(dy + row * hidden + c);
      const uint4 xr = *reinterpret_cast<const uint4*>(x + row * hidden + c);
      const __nv_bfloat16* dv = reinterpret_cast<const __nv_bfloat16*>(&dr);
      const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&xr);
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = __bfloat162float(dv[j]);
        const float xh = __bfloat162float(xv[j]) * r;
        o[j] = r * (d * w[c + j] - xh * s);
        mine[c + j] += d * xh;
      }
      uint4 out;
      out.x = pack2(o[0], o[1]);
      out.y = pack2(o[2], o[3]);
      out.z = pack2(o[4], o[5]);
      out.w = pack2(o[6], o[7]);
      *reinterpret_cast<uint4*>(dx + row * hidden + c) = out;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    float t = 0.f;
    for (int k = 0; k < kWarps; ++k) t += part[k * hidden + c];
    scratch[static_cast<int64_t>(blockIdx.x) * hidden + c] = t;
  }
}

// dweight[c] = sum over blocks of scratch[b, c], in block order (deterministic)
__global__ void rms_bwd_reduce(const float* __restrict__ scratch, int blocks, int hidden, float* __restrict__ dw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= hidden) return;
  float t = 0.f;
  for (int b = 0; b < blocks; ++b) t += scratch[static_cast<int64_t>(b) * hidden + c];
  dw[c] = t;
}

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
float* g_scratch[kMaxDevices] = {};
bool g_smem_configured[kMaxDevices] = {};

}  // namespace

extern "C" QW_NOALLOC_API int qw_rmsnorm_backward_noalloc(const void* dy, const void* x, const float* weight,
                                                          const float* rstd, void* dx, float* dweight,
                                                          long long rows, int hidden, void* stream) {
  if (!dy || !x || !weight || !rstd || !dx || !dweight || rows < 0 || hidden <= 0 || hidden % 8)
    return QW_NOALLOC_BAD_ARGUMENT;
  const auto misaligned = [](const void* p, uintptr_t to) { return reinterpret_cast<uintptr_t>(p) % to != 0; };
  if (misaligned(dy, 16) || misaligned(x, 16) || misaligned(dx, 16) || misaligned(weight, 4) ||
      misaligned(rstd, 4) || misaligned(dweight, 4))
    return QW_NOALLOC_BAD_ARGUMENT;
  const long long blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (blocks * static_cast<long long>(hidden) > QW_NOALLOC_SCRATCH_FLOATS) return QW_NOALLOC_TOO_LARGE;
  const size_t smem = static_cast<size_t>(kWarps) * hidden * sizeof(float);
  if (smem > 227 * 1024) return QW_NOALLOC_TOO_LARGE;
  if (cudaPeekAtLastError() != cudaSuccess) return QW_NOALLOC_PENDING_ERROR;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return QW_NOALLOC_CUDA_ERROR;
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch[device]) {
      // once per device, with that device current: the device address of this device's copy of the array
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, qw_noalloc_scratch) != cudaSuccess || !ptr) return QW_NOALLOC_CUDA_ERROR;
      g_scratch[device] = static_cast<float*>(ptr);
    }
    if (!g_smem_configured[device]) {
      if (cudaFuncSetAttribute(rms_bwd_partials, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(227 * 1024)) != cudaSuccess)
        return QW_NOALLOC_CUDA_ERROR;
      g_smem_configured[device] = true;
    }
    scratch = g_scratch[device];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (blocks > 0) {
    rms_bwd_partials<<<static_cast<unsigned>(blocks), kWarps * 32, smem, s>>>(
        static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), weight, rstd,
        static_cast<__nv_bfloat16*>(dx), scratch, rows, hidden);
    if (cudaGetLastError() != cudaSuccess) return QW_NOALLOC_CUDA_ERROR;  // nothing was pending on entry
  }
  rms_bwd_reduce<<<(hidden + 255) / 256, 256, 0, s>>>(scratch, static_cast<int>(blocks), hidden, dweight);
  return cudaGetLastError() == cudaSuccess ? QW_NOALLOC_OK : QW_NOALLOC_CUDA_ERROR;
}

extern "C" QW_NOALLOC_API const char* qw_noalloc_error_message(int code) {
  switch (code) {
    case QW_NOALLOC_OK: return "ok";
    case QW_NOALLOC_BAD_ARGUMENT:
      return "bad argument: null pointer, negative rows, hidden not a positive multiple of 8, dy/x/dx not 16-byte "
             "aligned, or weight/rstd/dweight not 4-byte aligned";
    case QW_NOALLOC_TOO_LARGE:
      return "problem too large: ceil(rows/256) * hidden exceeds the 4,194,304-float (16 MiB) static scratch array";
    case QW_NOALLOC_CUDA_ERROR: return "CUDA error during this call's set-up or launch (see cudaGetLastError)";
    case QW_NOALLOC_PENDING_ERROR:
      return "an earlier CUDA error is pending on this thread; nothing was launched and the error was left in place";
    default: return "unknown error code";
  }
}

extern "C" QW_NOALLOC_API long long qw_noalloc_scratch_floats() { return QW_NOALLOC_SCRATCH_FLOATS; }
