// RMSNorm / LayerNorm (forward with optional fused residual add, backward with fused residual-gradient add and
// deterministic two-stage weight-gradient reduction) and rotate-half RoPE on packed QKV rows.
//
// Layout: rows of `H` bf16 values, one warp per row; weights/biases and statistics in fp32.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

template <bool RMS>
__global__ void norm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ delta, bf16* __restrict__ x_out,
                                const float* __restrict__ w, const float* __restrict__ b, bf16* __restrict__ y,
                                float* __restrict__ mean_out, float* __restrict__ rstd_out, int64_t rows, int H,
                                float eps) {
  const int warps = blockDim.x / 32;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const bf16* xr = x + row * H;
  float sum = 0.f, sq = 0.f;
  // pass 1: statistics (values re-read in pass 2; rows are L1/L2 resident)
  for (int c = lane * 8; c < H; c += 256) {
    uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
    const bf16* v = reinterpret_cast<const bf16*>(&raw);
    uint4 draw;
    const bf16* dv = nullptr;
    if (delta) {
      draw = *reinterpret_cast<const uint4*>(delta + row * H + c);
      dv = reinterpret_cast<const bf16*>(&draw);
    }
    float vals[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = __bfloat162float(v[j]);
      if (delta) f = __bfloat162float(__float2bfloat16(f + __bfloat162float(dv[j])));
      vals[j] = f;
      sum += f;
      sq += f * f;
    }
    if (delta) {
      uint4 o;
      o.x = pack_bf16(vals[0], vals[1]); o.y = pack_bf16(vals[2], vals[3]);
      o.z = pack_bf16(vals[4], vals[5]); o.w = pack_bf16(vals[6], vals[7]);
      *reinterpret_cast<uint4*>(x_out + row * H + c) = o;
    }
  }
  sum = warp_sum(sum);
  sq = warp_sum(sq);
  float mean = 0.f, rstd;
  if (RMS) {
    rstd = rsqrtf(sq / H + eps);
  } else {
    mean = sum / H;
    const float var = fmaxf(sq / H - mean * mean, 0.f);
    rstd = rsqrtf(var + eps);
  }
  if (lane == 0) {
    rstd_out[row] = rstd;
    if (!RMS && mean_out) mean_out[row] = mean;
  }
  const bf16* src = delta ? x_out + row * H : xr;
  __syncwarp();
  for (int c = lane * 8; c < H; c += 256) {
    uint4 raw = *reinterpret_cast<const uint4*>(src + c);
    const bf16* v = reinterpret_cast<const bf16*>(&raw);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = (__bfloat162float(v[j]) - mean) * rstd * w[c + j];
      if (!RMS && b) f += b[c + j];
      o[j] = f;
    }
    uint4 out;
    out.x = pack_bf16(o[0], o[1]); out.y = pack_bf16(o[2], o[3]);
    out.z = pack_bf16(o[4], o[5]); out.w = pack_bf16(o[6], o[7]);
    *reinterpret_cast<uint4*>(y + row * H + c) = out;
  }
}

// dx = rstd * (w*dy - mean(w*dy) [LN only] - xhat * mean(w*dy*xhat)) (+ dres); partial dw/db per block
template <bool RMS>
__global__ void norm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x, const float* __restrict__ w,
                                const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                                const bf16* __restrict__ dres, bf16* __restrict__ dx, float* __restrict__ dw_part,
                                float* __restrict__ db_part, int64_t rows, int H, int rows_per_block) {
  extern __shared__ float sh[];  // [warps][H] dw partials then [warps][H] db partials
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  float* my_dw = sh + warp * H;
  float* my_db = sh + (warps + warp) * H;
  for (int c = lane; c < H; c += 32) {
    my_dw[c] = 0.f;
    if (!RMS) my_db[c] = 0.f;
  }
  __syncwarp();
  const int64_t first = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t last = min(rows, first + rows_per_block);
  for (int64_t row = first + warp; row < last; row += warps) {
    const float rstd = rstd_in[row];
    const float mean = RMS ? 0.f : mean_in[row];
    float s_g = 0.f, s_gx = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      uint4 dr = *reinterpret_cast<const uint4*>(dy + row * H + c);
      uint4 xr = *reinterpret_cast<const uint4*>(x + row * H + c);
      const bf16* dv = reinterpret_cast<const bf16*>(&dr);
      const bf16* xv = reinterpret_cast<const bf16*>(&xr);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g = __bfloat162float(dv[j]) * w[c + j];
        const float xh = (__bfloat162float(xv[j]) - mean) * rstd;
        s_g += g;
        s_gx += g * xh;
      }
    }
    s_g = warp_sum(s_g) / H;
    s_gx = warp_sum(s_gx) / H;
    for (int c = lane * 8; c < H; c += 256) {
      uint4 dr = *reinterpret_cast<const uint4*>(dy + row * H + c);
      uint4 xr = *reinterpret_cast<const uint4*>(x + row * H + c);
      const bf16* dv = reinterpret_cast<const bf16*>(&dr);
      const bf16* xv = reinterpret_cast<const bf16*>(&xr);
      float o[8];
      uint4 rr;
      const bf16* rv = nullptr;
      if (dres) {
        rr = *reinterpret_cast<const uint4*>(dres + row * H + c);
        rv = reinterpret_cast<const bf16*>(&rr);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = __bfloat162float(dv[j]);
        const float g = d * w[c + j];
        const float xh = (__bfloat162float(xv[j]) - mean) * rstd;
        float v = rstd * (g - (RMS ? 0.f : s_g) - xh * s_gx);
        if (dres) v += __bfloat162float(rv[j]);
        o[j] = v;
        my_dw[c + j] += d * xh;
        if (!RMS) my_db[c + j] += d;
      }
      uint4 out;
      out.x = pack_bf16(o[0], o[1]); out.y = pack_bf16(o[2], o[3]);
      out.z = pack_bf16(o[4], o[5]); out.w = pack_bf16(o[6], o[7]);
      *reinterpret_cast<uint4*>(dx + row * H + c) = out;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float s = 0.f, t = 0.f;
    for (int k = 0; k < warps; ++k) {
      s += sh[k * H + c];
      if (!RMS) t += sh[(warps + k) * H + c];
    }
    dw_part[static_cast<int64_t>(blockIdx.x) * H + c] = s;
    if (!RMS) db_part[static_cast<int64_t>(blockIdx.x) * H + c] = t;
  }
}

// out[c] (+)= sum_b part[b, c]   (fixed order: deterministic)
__global__ void column_sum_kernel(const float* __restrict__ part, int blocks, int H, float* __restrict__ out,
                                  bool accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int b = 0; b < blocks; ++b) s += part[static_cast<int64_t>(b) * H + c];
  out[c] = accumulate ? out[c] + s : s;
}

// Rotate-half RoPE in place on q and k heads of packed rows [T, (Hq + 2Hkv) * D]; position = row % seq
// (or positions[row] when given). sign = +1 forward, -1 backward (inverse rotation).
__global__ void rope_kernel(bf16* __restrict__ qkv, int64_t rows, int heads_rot, int D, int64_t ld, int seq,
                            const int* __restrict__ positions, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, float sign) {
  const int half = D / 2;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t per_row = static_cast<int64_t>(heads_rot) * half;
  if (idx >= rows * per_row) return;
  const int64_t row = idx / per_row;
  const int rem = static_cast<int>(idx % per_row);
  const int head = rem / half;
  const int i = rem % half;
  const int pos = positions ? positions[row] : static_cast<int>(row % seq);
  const float c = cos_t[static_cast<int64_t>(pos) * half + i];
  const float s = sign * sin_t[static_cast<int64_t>(pos) * half + i];
  bf16* p = qkv + row * ld + static_cast<int64_t>(head) * D;
  const float x1 = __bfloat162float(p[i]);
  const float x2 = __bfloat162float(p[i + half]);
  p[i] = __float2bfloat16(x1 * c - x2 * s);
  p[i + half] = __float2bfloat16(x2 * c + x1 * s);
}

}  // namespace

void norm_fwd(const bf16* x, const bf16* delta, bf16* x_out, const float* w, const float* b, bf16* y, float* mean,
              float* rstd, int64_t rows, int H, float eps, bool rms, cudaStream_t stream) {
  if (rows == 0) return;
  if (H % 8) throw std::runtime_error("norm: hidden size must be a multiple of 8");
  const int warps = 8;
  const int grid = static_cast<int>((rows + warps - 1) / warps);
  if (rms)
    norm_fwd_kernel<true><<<grid, warps * 32, 0, stream>>>(x, delta, x_out, w, b, y, mean, rstd, rows, H, eps);
  else
    norm_fwd_kernel<false><<<grid, warps * 32, 0, stream>>>(x, delta, x_out, w, b, y, mean, rstd, rows, H, eps);
  check_cuda(cudaGetLastError(), "norm_fwd");
}

int norm_bwd_blocks(int64_t rows) {
  const int64_t rpb = 256;
  return static_cast<int>(std::max<int64_t>(1, (rows + rpb - 1) / rpb));
}

void norm_bwd(const bf16* dy, const bf16* x, const float* w, const float* mean, const float* rstd, const bf16* dres,
              bf16* dx, float* dw_part, float* db_part, float* dw, float* db, int64_t rows, int H, bool rms,
              bool accumulate, cudaStream_t stream) {
  if (H % 8) throw std::runtime_error("norm: hidden size must be a multiple of 8");
  const int rpb = 256;
  const int blocks = norm_bwd_blocks(rows);
  const int warps = std::max(1, std::min(8, (200 * 1024) / (2 * H * static_cast<int>(sizeof(float)))));
  const size_t smem = static_cast<size_t>(2 * warps) * H * sizeof(float);
  if (rows > 0) {
    if (rms) {
      check_cuda(cudaFuncSetAttribute(norm_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                 "norm smem");
      norm_bwd_kernel<true><<<blocks, warps * 32, smem, stream>>>(dy, x, w, mean, rstd, dres, dx, dw_part, db_part, rows,
                                                                  H, rpb);
    } else {
      check_cuda(cudaFuncSetAttribute(norm_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                 "norm smem");
      norm_bwd_kernel<false><<<blocks, warps * 32, smem, stream>>>(dy, x, w, mean, rstd, dres, dx, dw_part, db_part,
                                                                   rows, H, rpb);
    }
    check_cuda(cudaGetLastError(), "norm_bwd");
  }
  const int actual_blocks = rows > 0 ? blocks : 0;
  if (actual_blocks == 0 && !accumulate) {
    cudaMemsetAsync(dw, 0, H * sizeof(float), stream);
    if (!rms && db) cudaMemsetAsync(db, 0, H * sizeof(float), stream);
    return;
  }
  column_sum_kernel<<<(H + 255) / 256, 256, 0, stream>>>(dw_part, actual_blocks, H, dw, accumulate);
  if (!rms && db) column_sum_kernel<<<(H + 255) / 256, 256, 0, stream>>>(db_part, actual_blocks, H, db, accumulate);
  check_cuda(cudaGetLastError(), "norm_bwd reduce");
}

void rope_apply(bf16* qkv, int64_t rows, int heads_rot, int D, int64_t ld, int seq, const int* positions,
                const float* cos_t, const float* sin_t, bool inverse, cudaStream_t stream) {
  const int64_t n = rows * heads_rot * (D / 2);
  if (n == 0) return;
  rope_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, stream>>>(qkv, rows, heads_rot, D, ld, seq, positions,
                                                                      cos_t, sin_t, inverse ? -1.f : 1.f);
  check_cuda(cudaGetLastError(), "rope");
}

int norm_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
