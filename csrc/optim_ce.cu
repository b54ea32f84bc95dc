// Fused multi-tensor AdamW (with fp32 master weights, the gradient-norm clip folded in) and the cross-entropy
// kernel used by the chunked linear-cross-entropy.
//
// AdamW follows torch.optim.AdamW's update exactly (decoupled decay, bias-corrected moments):
//   p <- p * (1 - lr*wd);  m <- b1*m + (1-b1)*g;  v <- b2*v + (1-b2)*g^2
//   p <- p - (lr / (1-b1^t)) * m / (sqrt(v) / sqrt(1-b2^t) + eps)
// with g = grad * clip_coef, clip_coef = min(1, max_norm / (||grad||_2 + 1e-6)) computed on the device from a
// fixed-order (deterministic) sum of squares.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

constexpr int kAdamChunk = 8192;

__device__ __forceinline__ float load_val(const void* p, int64_t i, int dtype) {
  return dtype == 0 ? static_cast<const float*>(p)[i] : __bfloat162float(static_cast<const bf16*>(p)[i]);
}

__device__ __forceinline__ void load4(const void* p, int64_t i, int dtype, float* g) {
  if (dtype == 0) {
    const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    g[0] = v.x; g[1] = v.y; g[2] = v.z; g[3] = v.w;
  } else {
    const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const bf16*>(p) + i);
    const bf16* b = reinterpret_cast<const bf16*>(&raw);
    g[0] = __bfloat162float(b[0]); g[1] = __bfloat162float(b[1]);
    g[2] = __bfloat162float(b[2]); g[3] = __bfloat162float(b[3]);
  }
}

__device__ __forceinline__ bool vec_ok(const AdamTensor& t) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(t.param) | reinterpret_cast<uintptr_t>(t.grad) |
                         reinterpret_cast<uintptr_t>(t.exp_avg) | reinterpret_cast<uintptr_t>(t.exp_avg_sq) |
                         reinterpret_cast<uintptr_t>(t.master);
  return (bits & 15) == 0 && (t.numel & 3) == 0;
}

// partial[chunk] = sum of squares of the chunk's (scaled) gradient elements
__global__ void sumsq_kernel(const AdamTensor* __restrict__ tensors, const int* __restrict__ chunk_tensor,
                             const int64_t* __restrict__ chunk_start, double* __restrict__ partial) {
  const int chunk = blockIdx.x;
  const AdamTensor& t = tensors[chunk_tensor[chunk]];
  const int64_t begin = chunk_start[chunk];
  const int64_t end = min(t.numel, begin + kAdamChunk);
  float s = 0.f;
  if (vec_ok(t)) {
    for (int64_t i = begin + 4 * threadIdx.x; i < end; i += 4 * blockDim.x) {
      float g[4];
      load4(t.grad, i, t.grad_dtype, g);
#pragma unroll
      for (int j = 0; j < 4; ++j) s += (g[j] * t.grad_scale) * (g[j] * t.grad_scale);
    }
  } else {
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
      const float g = load_val(t.grad, i, t.grad_dtype) * t.grad_scale;
      s += g * g;
    }
  }
  __shared__ float red[32];
  s = warp_sum(s);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double acc = 0.0;
    for (int w = 0; w < blockDim.x / 32; ++w) acc += red[w];
    partial[chunk] = acc;
  }
}

// norm_out[0] = ||g||, norm_out[1] = clip coefficient (fixed-order sum over chunks)
__global__ void norm_finalize_kernel(const double* __restrict__ partial, int chunks, float max_norm,
                                     const double* __restrict__ extra_sumsq, float* __restrict__ norm_out) {
  __shared__ double red[1024];
  double s = 0.0;
  for (int i = threadIdx.x; i < chunks; i += blockDim.x) s += partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double total = 0.0;
    for (int i = 0; i < blockDim.x; ++i) total += red[i];
    if (extra_sumsq) total += extra_sumsq[0];
    const double norm = sqrt(total);
    norm_out[0] = static_cast<float>(norm);
    norm_out[1] = max_norm > 0.f ? static_cast<float>(fmin(1.0, max_norm / (norm + 1e-6))) : 1.f;
  }
}

__device__ __forceinline__ void adam_update(float& p, float& m, float& v, float g, const AdamHyper& h, float decay,
                                            float step_size) {
  p *= decay;
  m = h.beta1 * m + (1.f - h.beta1) * g;
  v = h.beta2 * v + (1.f - h.beta2) * g * g;
  const float denom = sqrtf(v) / h.bias_correction2_sqrt + h.eps;
  p -= step_size * m / denom;
}

// Small-footprint variant for an update that runs beside other kernels (the optimizer overlapped with the next
// forward): 128-thread blocks, a grid of a couple of blocks per SM striding over the chunks, two 4-element groups
// in flight per thread. A block fits next to a persistent GEMM or attention CTA (registers and threads to spare,
// no shared memory), so the update streams through HBM while those kernels run.
__device__ __forceinline__ void adamw_chunk_small(const AdamTensor& t, int64_t begin, AdamHyper h, float coef) {
  const int64_t end = min(t.numel, begin + kAdamChunk);
  const float decay = 1.f - h.lr * h.weight_decay * t.decay_scale;
  const float step_size = h.lr / h.bias_correction1;
  float* master = t.master ? t.master : static_cast<float*>(t.param);
  if (vec_ok(t)) {
    for (int64_t i0 = begin + 4 * threadIdx.x; i0 < end; i0 += 8 * blockDim.x) {
      float g[2][4];
      float4 p[2], m[2], v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t i = i0 + u * 4 * blockDim.x;
        if (i >= end) break;
        load4(t.grad, i, t.grad_dtype, g[u]);
        p[u] = *reinterpret_cast<const float4*>(master + i);
        m[u] = *reinterpret_cast<const float4*>(t.exp_avg + i);
        v[u] = *reinterpret_cast<const float4*>(t.exp_avg_sq + i);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t i = i0 + u * 4 * blockDim.x;
        if (i >= end) break;
        adam_update(p[u].x, m[u].x, v[u].x, g[u][0] * coef, h, decay, step_size);
        adam_update(p[u].y, m[u].y, v[u].y, g[u][1] * coef, h, decay, step_size);
        adam_update(p[u].z, m[u].z, v[u].z, g[u][2] * coef, h, decay, step_size);
        adam_update(p[u].w, m[u].w, v[u].w, g[u][3] * coef, h, decay, step_size);
        *reinterpret_cast<float4*>(master + i) = p[u];
        *reinterpret_cast<float4*>(t.exp_avg + i) = m[u];
        *reinterpret_cast<float4*>(t.exp_avg_sq + i) = v[u];
        if (t.master) {
          uint2 out;
          out.x = pack_bf16(p[u].x, p[u].y);
          out.y = pack_bf16(p[u].z, p[u].w);
          *reinterpret_cast<uint2*>(static_cast<bf16*>(t.param) + i) = out;
        }
      }
    }
  } else {
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
      float p = master[i], m = t.exp_avg[i], v = t.exp_avg_sq[i];
      adam_update(p, m, v, load_val(t.grad, i, t.grad_dtype) * coef, h, decay, step_size);
      master[i] = p;
      t.exp_avg[i] = m;
      t.exp_avg_sq[i] = v;
      if (t.master) static_cast<bf16*>(t.param)[i] = __float2bfloat16(p);
    }
  }
}

__global__ void __launch_bounds__(128, 4) adamw_small_kernel(const AdamTensor* __restrict__ tensors,
                                                             const int* __restrict__ chunk_tensor,
                                                             const int64_t* __restrict__ chunk_start, int chunks,
                                                             AdamHyper h, const float* __restrict__ clip) {
  for (int chunk = blockIdx.x; chunk < chunks; chunk += gridDim.x) {
    const AdamTensor& t = tensors[chunk_tensor[chunk]];
    adamw_chunk_small(t, chunk_start[chunk], h, (clip ? clip[1] : 1.f) * t.grad_scale);
  }
}

__global__ void adamw_kernel(const AdamTensor* __restrict__ tensors, const int* __restrict__ chunk_tensor,
                             const int64_t* __restrict__ chunk_start, AdamHyper h, const float* __restrict__ clip) {
  const int chunk = blockIdx.x;
  const AdamTensor& t = tensors[chunk_tensor[chunk]];
  const int64_t begin = chunk_start[chunk];
  const int64_t end = min(t.numel, begin + kAdamChunk);
  const float coef = (clip ? clip[1] : 1.f) * t.grad_scale;
  const float decay = 1.f - h.lr * h.weight_decay * t.decay_scale;
  const float step_size = h.lr / h.bias_correction1;
  float* master = t.master ? t.master : static_cast<float*>(t.param);
  if (vec_ok(t)) {
    for (int64_t i = begin + 4 * threadIdx.x; i < end; i += 4 * blockDim.x) {
      float g[4];
      load4(t.grad, i, t.grad_dtype, g);
      float4 p = *reinterpret_cast<const float4*>(master + i);
      float4 m = *reinterpret_cast<const float4*>(t.exp_avg + i);
      float4 v = *reinterpret_cast<const float4*>(t.exp_avg_sq + i);
      adam_update(p.x, m.x, v.x, g[0] * coef, h, decay, step_size);
      adam_update(p.y, m.y, v.y, g[1] * coef, h, decay, step_size);
      adam_update(p.z, m.z, v.z, g[2] * coef, h, decay, step_size);
      adam_update(p.w, m.w, v.w, g[3] * coef, h, decay, step_size);
      *reinterpret_cast<float4*>(master + i) = p;
      *reinterpret_cast<float4*>(t.exp_avg + i) = m;
      *reinterpret_cast<float4*>(t.exp_avg_sq + i) = v;
      if (t.master) {
        uint2 out;
        out.x = pack_bf16(p.x, p.y);
        out.y = pack_bf16(p.z, p.w);
        *reinterpret_cast<uint2*>(static_cast<bf16*>(t.param) + i) = out;
      }
    }
  } else {
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
      float p = master[i], m = t.exp_avg[i], v = t.exp_avg_sq[i];
      adam_update(p, m, v, load_val(t.grad, i, t.grad_dtype) * coef, h, decay, step_size);
      master[i] = p;
      t.exp_avg[i] = m;
      t.exp_avg_sq[i] = v;
      if (t.master) static_cast<bf16*>(t.param)[i] = __float2bfloat16(p);
    }
  }
}

// 8-bit moments: the state of a tensor is one byte buffer [m: int8 x P][sqrt v: uint8 x P][scales: fp32 x 2 per
// 2048-element block], P = numel rounded up to 16; exp_avg points at its start and exp_avg_sq at the second part.
// m is stored linearly against its block absmax (127 levels each side), sqrt(v) linearly against its block max (255
// levels): block-wise quantisation of the optimiser state. The update itself runs in fp32 on the dequantised values;
// the new block scales come from a block reduction before re-quantising.
constexpr int kQBlock = 2048;

__global__ void __launch_bounds__(256) adamw8_kernel(const AdamTensor* __restrict__ tensors,
                                                     const int* __restrict__ chunk_tensor,
                                                     const int64_t* __restrict__ chunk_start, AdamHyper h,
                                                     const float* __restrict__ clip) {
  __shared__ float red_m[8], red_v[8];
  const AdamTensor& t = tensors[chunk_tensor[blockIdx.x]];
  const int64_t begin = chunk_start[blockIdx.x];
  const int64_t end = min(t.numel, begin + kAdamChunk);
  const int64_t padded = (t.numel + 15) / 16 * 16;
  int8_t* mq = static_cast<int8_t*>(static_cast<void*>(t.exp_avg));
  uint8_t* vq = static_cast<uint8_t*>(static_cast<void*>(t.exp_avg_sq));
  float* scales = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(t.exp_avg) + 2 * padded);
  const float coef = (clip ? clip[1] : 1.f) * t.grad_scale;
  const float decay = 1.f - h.lr * h.weight_decay * t.decay_scale;
  const float step_size = h.lr / h.bias_correction1;
  float* master = t.master ? t.master : static_cast<float*>(t.param);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int64_t b0 = begin; b0 < end; b0 += kQBlock) {
    const int64_t qb = b0 / kQBlock;
    const float sm_old = scales[2 * qb], sv_old = scales[2 * qb + 1];
    float m[8], v[8];
    float amax_m = 0.f, amax_v = 0.f;
    const int64_t i0 = b0 + threadIdx.x * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = i0 + j;
      m[j] = v[j] = 0.f;
      if (i >= end) continue;
      const float g = load_val(t.grad, i, t.grad_dtype) * coef;
      const float root = static_cast<float>(vq[i]) * sv_old;
      float mm = h.beta1 * (static_cast<float>(mq[i]) * sm_old) + (1.f - h.beta1) * g;
      float vv = h.beta2 * (root * root) + (1.f - h.beta2) * g * g;
      float p = master[i] * decay;
      p -= step_size * mm / (sqrtf(vv) / h.bias_correction2_sqrt + h.eps);
      master[i] = p;
      if (t.master) static_cast<bf16*>(t.param)[i] = __float2bfloat16(p);
      m[j] = mm;
      v[j] = sqrtf(vv);
      amax_m = fmaxf(amax_m, fabsf(mm));
      amax_v = fmaxf(amax_v, v[j]);
    }
    amax_m = warp_max(amax_m);
    amax_v = warp_max(amax_v);
    if (lane == 0) {
      red_m[warp] = amax_m;
      red_v[warp] = amax_v;
    }
    __syncthreads();
    amax_m = 0.f;
    amax_v = 0.f;
    for (int w = 0; w < blockDim.x / 32; ++w) {
      amax_m = fmaxf(amax_m, red_m[w]);
      amax_v = fmaxf(amax_v, red_v[w]);
    }
    const float inv_m = amax_m > 0.f ? 127.f / amax_m : 0.f;
    const float inv_v = amax_v > 0.f ? 255.f / amax_v : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = i0 + j;
      if (i >= end) continue;
      mq[i] = static_cast<int8_t>(fminf(127.f, fmaxf(-127.f, rintf(m[j] * inv_m))));
      vq[i] = static_cast<uint8_t>(fminf(255.f, rintf(v[j] * inv_v)));
    }
    if (threadIdx.x == 0) {
      scales[2 * qb] = amax_m / 127.f;
      scales[2 * qb + 1] = amax_v / 255.f;
    }
    __syncthreads();
  }
}

// in-place per-row cross-entropy gradient on a logits chunk; loss_out[row] = lse - logit[label] (0 if ignored)
__global__ void __launch_bounds__(256) ce_kernel(bf16* __restrict__ logits, int64_t ld, int V,
                                                 const int64_t* __restrict__ labels, float grad_scale,
                                                 float* __restrict__ loss_out, int ignore_index) {
  const int64_t row = blockIdx.x;
  bf16* l = logits + row * ld;
  const int64_t label = labels[row];
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = __bfloat162float(l[i]);
    if (x > m) {
      s = s * __expf(m - x) + 1.f;
      m = x;
    } else {
      s += __expf(x - m);
    }
  }
  __shared__ float sm[32], ss[32];
  // warp combine of (m, s)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  if (threadIdx.x % 32 == 0) { sm[threadIdx.x / 32] = m; ss[threadIdx.x / 32] = s; }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x / 32;
    m = threadIdx.x < nw ? sm[threadIdx.x] : -INFINITY;
    s = threadIdx.x < nw ? ss[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (threadIdx.x == 0) { sm[0] = m; ss[0] = s; }
  }
  __syncthreads();
  m = sm[0];
  s = ss[0];
  const bool ignored = (label == ignore_index);
  const float lse = m + __logf(s);
  if (threadIdx.x == 0) loss_out[row] = ignored ? 0.f : lse - __bfloat162float(l[label]);
  __syncthreads();
  const float inv_s = 1.f / s;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float g = 0.f;
    if (!ignored) {
      g = __expf(__bfloat162float(l[i]) - m) * inv_s;
      if (i == label) g -= 1.f;
      g *= grad_scale;
    }
    l[i] = __float2bfloat16(g);
  }
}

// Register-resident variant for rows of at most 8 * 256 * CPT columns (16-byte aligned rows, V a multiple of 8): the
// row is read once with 16-byte loads and kept in registers, the maximum and the sum of exponentials are block
// reductions over it, and the gradient is written back with 16-byte stores. One read and one write per element,
// against two reads, one write and a data-dependent branch per element in ce_kernel above.
template <int CPT>
__global__ void __launch_bounds__(256) ce_row_kernel(bf16* __restrict__ logits, int64_t ld, int V,
                                                     const int64_t* __restrict__ labels, float grad_scale,
                                                     float* __restrict__ loss_out, int ignore_index) {
  constexpr float kLog2e = 1.4426950408889634f;
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  bf16* l = logits + row * ld;
  const int64_t label = labels[row];
  const int chunks = V / 8;
  uint4 raw[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    const int i = threadIdx.x + c * 256;
    raw[c] = i < chunks ? reinterpret_cast<const uint4*>(l)[i] : make_uint4(0, 0, 0, 0);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  auto block_reduce = [&](float v, bool is_max) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, w) : v + w;
    }
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
    __syncthreads();  // red is reused by the next reduction
    return r;
  };
  float m = -INFINITY;
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    if (threadIdx.x + c * 256 >= chunks) break;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[c]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      m = fmax3(m, f.x, f.y);
    }
  }
  m = block_reduce(m, true);
  const float ml2 = m * kLog2e;
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    if (threadIdx.x + c * 256 >= chunks) break;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[c]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      s += exp2f_approx(fmaf(f.x, kLog2e, -ml2)) + exp2f_approx(fmaf(f.y, kLog2e, -ml2));
    }
  }
  s = block_reduce(s, false);
  const bool ignored = (label == ignore_index);
  if (threadIdx.x == 0) loss_out[row] = ignored ? 0.f : m + __logf(s) - __bfloat162float(l[label]);
  const float scale = ignored ? 0.f : grad_scale / s;
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    const int i = threadIdx.x + c * 256;
    if (i >= chunks) break;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[c]);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      float g0 = exp2f_approx(fmaf(f.x, kLog2e, -ml2)) * scale;
      float g1 = exp2f_approx(fmaf(f.y, kLog2e, -ml2)) * scale;
      const int64_t col = 8 * static_cast<int64_t>(i) + 2 * j;
      if (!ignored && col == label) g0 -= grad_scale;
      if (!ignored && col + 1 == label) g1 -= grad_scale;
      o[j] = pack_bf16(g0, g1);
    }
    reinterpret_cast<uint4*>(l)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void scale_bf16_kernel(bf16* __restrict__ x, int64_t n, const float* __restrict__ scale) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __float2bfloat16(__bfloat162float(x[i]) * scale[0]);
}

}  // namespace

int adam_chunk_size() { return kAdamChunk; }
int adam8_block_size() { return kQBlock; }

void adam_grad_norm(const AdamTensor* tensors, const int* chunk_tensor, const int64_t* chunk_start, int chunks,
                    double* partial, const double* extra_sumsq, float max_norm, float* norm_out, cudaStream_t stream) {
  if (chunks > 0) sumsq_kernel<<<chunks, 256, 0, stream>>>(tensors, chunk_tensor, chunk_start, partial);
  norm_finalize_kernel<<<1, 1024, 0, stream>>>(partial, chunks, max_norm, extra_sumsq, norm_out);
  check_cuda(cudaGetLastError(), "adam_grad_norm");
}

void adam_sumsq(const AdamTensor* tensors, const int* chunk_tensor, const int64_t* chunk_start, int chunks,
                double* partial, cudaStream_t stream) {
  if (chunks > 0) sumsq_kernel<<<chunks, 256, 0, stream>>>(tensors, chunk_tensor, chunk_start, partial);
  check_cuda(cudaGetLastError(), "adam_sumsq");
}

void adam_step(const AdamTensor* tensors, const int* chunk_tensor, const int64_t* chunk_start, int chunks,
               const AdamHyper& hyper, const float* clip, bool eight_bit, cudaStream_t stream, int small_blocks) {
  if (chunks == 0) return;
  if (small_blocks > 0 && !eight_bit)
    adamw_small_kernel<<<std::min(chunks, small_blocks), 128, 0, stream>>>(tensors, chunk_tensor, chunk_start, chunks,
                                                                          hyper, clip);
  else if (eight_bit)
    adamw8_kernel<<<chunks, 256, 0, stream>>>(tensors, chunk_tensor, chunk_start, hyper, clip);
  else
    adamw_kernel<<<chunks, 256, 0, stream>>>(tensors, chunk_tensor, chunk_start, hyper, clip);
  check_cuda(cudaGetLastError(), "adam_step");
}

void cross_entropy_chunk(bf16* logits, int64_t rows, int64_t ld, int V, const int64_t* labels, float grad_scale,
                         float* loss_out, int ignore_index, cudaStream_t stream) {
  if (rows == 0) return;
  const bool vec = V % 8 == 0 && (ld * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  if (vec && V <= 8 * 256 * 8) {
    ce_row_kernel<8><<<static_cast<int>(rows), 256, 0, stream>>>(logits, ld, V, labels, grad_scale, loss_out,
                                                                 ignore_index);
  } else if (vec && V <= 8 * 256 * 16) {
    ce_row_kernel<16><<<static_cast<int>(rows), 256, 0, stream>>>(logits, ld, V, labels, grad_scale, loss_out,
                                                                  ignore_index);
  } else {
    ce_kernel<<<static_cast<int>(rows), 256, 0, stream>>>(logits, ld, V, labels, grad_scale, loss_out, ignore_index);
  }
  check_cuda(cudaGetLastError(), "cross_entropy_chunk");
}

void scale_bf16(bf16* x, int64_t n, const float* scale, cudaStream_t stream) {
  if (n == 0) return;
  scale_bf16_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, stream>>>(x, n, scale);
  check_cuda(cudaGetLastError(), "scale_bf16");
}

int optim_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
