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

__global__ void scale_bf16_kernel(bf16* __restrict__ x, int64_t n, const float* __restrict__ scale) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __float2bfloat16(__bfloat162float(x[i]) * scale[0]);
}

}  // namespace

int adam_chunk_size() { return kAdamChunk; }

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
               const AdamHyper& hyper, const float* clip, cudaStream_t stream) {
  if (chunks == 0) return;
  adamw_kernel<<<chunks, 256, 0, stream>>>(tensors, chunk_tensor, chunk_start, hyper, clip);
  check_cuda(cudaGetLastError(), "adam_step");
}

void cross_entropy_chunk(bf16* logits, int64_t rows, int64_t ld, int V, const int64_t* labels, float grad_scale,
                         float* loss_out, int ignore_index, cudaStream_t stream) {
  if (rows == 0) return;
  ce_kernel<<<static_cast<int>(rows), 256, 0, stream>>>(logits, ld, V, labels, grad_scale, loss_out, ignore_index);
  check_cuda(cudaGetLastError(), "cross_entropy_chunk");
}

void scale_bf16(bf16* x, int64_t n, const float* scale, cudaStream_t stream) {
  if (n == 0) return;
  scale_bf16_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, stream>>>(x, n, scale);
  check_cuda(cudaGetLastError(), "scale_bf16");
}

int optim_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
