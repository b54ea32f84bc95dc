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

// Register-resident variants for H = CH * 256 (CH <= 4): one warp per row, lane l owns columns l*8 + 256*k. The row,
// the weights and (backward) the dw/db accumulators stay in registers, so each element is read from HBM once and
// the weight gradient is accumulated without shared-memory traffic; the variance is computed around the mean.
template <bool RMS, int CH>
__global__ void __launch_bounds__(256) norm_fwd_reg_kernel(const bf16* __restrict__ x, const bf16* __restrict__ delta,
                                                           bf16* __restrict__ x_out, const float* __restrict__ w,
                                                           const float* __restrict__ b, bf16* __restrict__ y,
                                                           float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                           int64_t rows, float eps) {
  constexpr int H = CH * 256;
  const int lane = threadIdx.x % 32;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  float v[CH][8];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = lane * 8 + k * 256;
    const uint4 raw = *reinterpret_cast<const uint4*>(x + row * H + c);
    const bf16* xv = reinterpret_cast<const bf16*>(&raw);
    uint4 draw = make_uint4(0, 0, 0, 0);
    if (delta) draw = *reinterpret_cast<const uint4*>(delta + row * H + c);
    const bf16* dv = reinterpret_cast<const bf16*>(&draw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f = __bfloat162float(xv[j]);
      if (delta) f = __bfloat162float(__float2bfloat16(f + __bfloat162float(dv[j])));
      v[k][j] = f;
      sum += f;
    }
    if (delta) {
      uint4 o;
      o.x = pack_bf16(v[k][0], v[k][1]); o.y = pack_bf16(v[k][2], v[k][3]);
      o.z = pack_bf16(v[k][4], v[k][5]); o.w = pack_bf16(v[k][6], v[k][7]);
      *reinterpret_cast<uint4*>(x_out + row * H + c) = o;
    }
  }
  const float mean = RMS ? 0.f : warp_sum(sum) / H;
  float sq = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = v[k][j] - mean;
      sq += d * d;
    }
  const float rstd = rsqrtf(warp_sum(sq) / H + eps);
  if (lane == 0) {
    rstd_out[row] = rstd;
    if (!RMS && mean_out) mean_out[row] = mean;
  }
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = lane * 8 + k * 256;
    const float4 w0 = *reinterpret_cast<const float4*>(w + c);
    const float4 w1 = *reinterpret_cast<const float4*>(w + c + 4);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float bv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (!RMS && b) {
      const float4 b0 = *reinterpret_cast<const float4*>(b + c);
      const float4 b1 = *reinterpret_cast<const float4*>(b + c + 4);
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w; bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
    }
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = (v[k][j] - mean) * rstd * wv[j] + bv[j];
    uint4 out;
    out.x = pack_bf16(o[0], o[1]); out.y = pack_bf16(o[2], o[3]);
    out.z = pack_bf16(o[4], o[5]); out.w = pack_bf16(o[6], o[7]);
    *reinterpret_cast<uint4*>(y + row * H + c) = out;
  }
}

template <bool RMS, int CH>
__global__ void __launch_bounds__(256, 2) norm_bwd_reg_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                           const float* __restrict__ w,
                                                           const float* __restrict__ mean_in,
                                                           const float* __restrict__ rstd_in,
                                                           const bf16* __restrict__ dres, bf16* __restrict__ dx,
                                                           float* __restrict__ dw_part, float* __restrict__ db_part,
                                                           int64_t rows, int rows_per_block) {
  constexpr int H = CH * 256;
  extern __shared__ float red[];  // [warps][H]
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float acc_w[CH][8], acc_b[CH][8];
#pragma unroll
  for (int k = 0; k < CH; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc_w[k][j] = acc_b[k][j] = 0.f;
  auto load_w = [&](int c, float* out) {  // weights stay in L1; reloading is cheaper than holding them
    const float4 w0 = *reinterpret_cast<const float4*>(w + c);
    const float4 w1 = *reinterpret_cast<const float4*>(w + c + 4);
    out[0] = w0.x; out[1] = w0.y; out[2] = w0.z; out[3] = w0.w; out[4] = w1.x; out[5] = w1.y; out[6] = w1.z; out[7] = w1.w;
  };
  const int64_t first = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t last = min(rows, first + rows_per_block);
  for (int64_t row = first + warp; row < last; row += warps) {
    const float rstd = rstd_in[row];
    const float mean = RMS ? 0.f : mean_in[row];
    uint4 draw[CH], xraw[CH];
    float s_g = 0.f, s_gx = 0.f;
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const int c = lane * 8 + k * 256;
      draw[k] = *reinterpret_cast<const uint4*>(dy + row * H + c);
      xraw[k] = *reinterpret_cast<const uint4*>(x + row * H + c);
    }
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const bf16* dv = reinterpret_cast<const bf16*>(&draw[k]);
      const bf16* xv = reinterpret_cast<const bf16*>(&xraw[k]);
      float wv[8];
      load_w(lane * 8 + k * 256, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = __bfloat162float(dv[j]);
        const float g = d * wv[j];
        const float xh = (__bfloat162float(xv[j]) - mean) * rstd;
        s_g += g;
        s_gx += g * xh;
        acc_w[k][j] += d * xh;
        if (!RMS) acc_b[k][j] += d;
      }
    }
    s_g = warp_sum(s_g) / H;
    s_gx = warp_sum(s_gx) / H;
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const int c = lane * 8 + k * 256;
      const bf16* dv = reinterpret_cast<const bf16*>(&draw[k]);
      const bf16* xv = reinterpret_cast<const bf16*>(&xraw[k]);
      uint4 rr = make_uint4(0, 0, 0, 0);
      if (dres) rr = *reinterpret_cast<const uint4*>(dres + row * H + c);
      const bf16* rv = reinterpret_cast<const bf16*>(&rr);
      float wv[8];
      load_w(c, wv);
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g = __bfloat162float(dv[j]) * wv[j];
        const float xh = (__bfloat162float(xv[j]) - mean) * rstd;
        float val = rstd * (g - (RMS ? 0.f : s_g) - xh * s_gx);
        if (dres) val += __bfloat162float(rv[j]);
        o[j] = val;
      }
      uint4 out;
      out.x = pack_bf16(o[0], o[1]); out.y = pack_bf16(o[2], o[3]);
      out.z = pack_bf16(o[4], o[5]); out.w = pack_bf16(o[6], o[7]);
      *reinterpret_cast<uint4*>(dx + row * H + c) = out;
    }
  }
  // fixed-order reduction of the warps' register partials: dw, then db
#pragma unroll
  for (int pass = 0; pass < (RMS ? 1 : 2); ++pass) {
#pragma unroll
    for (int k = 0; k < CH; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp * H + lane * 8 + k * 256 + j] = pass == 0 ? acc_w[k][j] : acc_b[k][j];
    __syncthreads();
    float* out = pass == 0 ? dw_part : db_part;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
      float s = 0.f;
      for (int q = 0; q < warps; ++q) s += red[q * H + c];
      out[static_cast<int64_t>(blockIdx.x) * H + c] = s;
    }
    __syncthreads();
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

// Bias gradient, stage 1: part[slab, c] = sum of g[r, c] over the slab's rows (fp32). 64 threads x 8 columns per
// block, one uint4 load per thread per row; stage 2 is column_sum_kernel over the slabs (fixed order).
__global__ void __launch_bounds__(64) bias_grad_kernel(const bf16* __restrict__ g, int64_t ldg, int64_t rows, int N,
                                                       int rows_per_slab, float* __restrict__ part) {
  const int c = (blockIdx.x * 64 + threadIdx.x) * 8;
  if (c >= N) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_slab;
  const int64_t r1 = min(rows, r0 + rows_per_slab);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int64_t r = r0; r < r1; ++r) {
    const uint4 raw = *reinterpret_cast<const uint4*>(g + r * ldg + c);
    const bf16* v = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(v[j]);
  }
  float* out = part + static_cast<int64_t>(blockIdx.y) * N + c;
#pragma unroll
  for (int j = 0; j < 8; ++j) out[j] = acc[j];
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
  if (H % 256 == 0 && H <= 1024) {
#define QW_NF(R, C) norm_fwd_reg_kernel<R, C><<<grid, warps * 32, 0, stream>>>(x, delta, x_out, w, b, y, mean, rstd, rows, eps)
    const int ch = H / 256;
    if (rms) { if (ch == 1) QW_NF(true, 1); else if (ch == 2) QW_NF(true, 2); else if (ch == 3) QW_NF(true, 3); else QW_NF(true, 4); }
    else { if (ch == 1) QW_NF(false, 1); else if (ch == 2) QW_NF(false, 2); else if (ch == 3) QW_NF(false, 3); else QW_NF(false, 4); }
#undef QW_NF
    check_cuda(cudaGetLastError(), "norm_fwd");
    return;
  }
  if (rms)
    norm_fwd_kernel<true><<<grid, warps * 32, 0, stream>>>(x, delta, x_out, w, b, y, mean, rstd, rows, H, eps);
  else
    norm_fwd_kernel<false><<<grid, warps * 32, 0, stream>>>(x, delta, x_out, w, b, y, mean, rstd, rows, H, eps);
  check_cuda(cudaGetLastError(), "norm_fwd");
}

int bias_grad_slabs(int64_t rows) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(256, rows / 256))); }

void bias_grad(const bf16* g, int64_t ldg, int64_t rows, int N, float* part, float* out, bool accumulate,
               cudaStream_t stream) {
  if (N % 8 || ldg % 8) throw std::runtime_error("bias_grad: columns must be a multiple of 8");
  if (rows == 0) {
    if (!accumulate) cudaMemsetAsync(out, 0, N * sizeof(float), stream);
    return;
  }
  const int slabs = bias_grad_slabs(rows);
  const int per = static_cast<int>((rows + slabs - 1) / slabs);
  dim3 grid((N / 8 + 63) / 64, slabs);
  bias_grad_kernel<<<grid, 64, 0, stream>>>(g, ldg, rows, N, per, part);
  column_sum_kernel<<<(N + 255) / 256, 256, 0, stream>>>(part, slabs, N, out, accumulate);
  check_cuda(cudaGetLastError(), "bias_grad");
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
  if (rows > 0 && H % 256 == 0 && H <= 1024) {
    const size_t rsmem = static_cast<size_t>(8) * H * sizeof(float);
#define QW_NB(R, C)                                                                                                 \
  do {                                                                                                              \
    check_cuda(cudaFuncSetAttribute(norm_bwd_reg_kernel<R, C>, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                    int(rsmem)), "norm smem");                                                      \
    norm_bwd_reg_kernel<R, C><<<blocks, 256, rsmem, stream>>>(dy, x, w, mean, rstd, dres, dx, dw_part, db_part,   \
                                                              rows, rpb);                                           \
  } while (0)
    const int ch = H / 256;
    if (rms) { if (ch == 1) QW_NB(true, 1); else if (ch == 2) QW_NB(true, 2); else if (ch == 3) QW_NB(true, 3); else QW_NB(true, 4); }
    else { if (ch == 1) QW_NB(false, 1); else if (ch == 2) QW_NB(false, 2); else if (ch == 3) QW_NB(false, 3); else QW_NB(false, 4); }
#undef QW_NB
    check_cuda(cudaGetLastError(), "norm_bwd");
  } else if (rows > 0) {
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
