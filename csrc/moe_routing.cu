// MoE routing on the device, with no host synchronisation:
//
//   router logits   fp32 SIMT GEMM  logits[T,E] = x[T,H] . Wr[E,H]^T          (router stays fp32, as in the reference)
//   topk            softmax(logits / temperature), top-k by probability (or by logits + expert_bias), renormalised
//                   weights, per-expert route counts
//   plan            capacity cut: kept = min(count, cap); expert segments padded to 128 rows; overflow total
//   rank            stable counting sort of routes by expert (route order inside an expert)
//   select          experts over capacity keep their `cap` routes with the largest (weight, -route) key: an exact
//                   radix select on 64-bit keys, then an order-preserving compaction
//   permute         x_perm[row] = x[token], zero padding rows; row -> token / weight maps
//   combine         out[t] = resid[t] + sum_j w_j * y[row(t, j)]   (fixed j order: deterministic, no atomics)
//   backward        row gathers, per-route weight gradient reduction, softmax/renormalisation backward,
//                   router input/weight gradients (SIMT GEMMs, split-K with a fixed-order reduction)
//
// Reference behaviour: src/quantweave_moe_model.py:113-188 (route ordering by expert then weight, capacity).
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

// ------------------------------------------------------------------------------------------------ SIMT GEMM
// C[M,N] (+)= alpha * sum_k A[m,k] * B[k,n], generic strides, fp32 accumulate; split-K along gridDim.z writes
// partial slabs C + z*M*N (reduced by a fixed-order kernel).
// C[M,N] (+)= alpha * A[M,K] . B[K,N], fp32 FMA (the router runs in fp32). 64x64 tile, BK = 32, 256 threads with 4x4
// outputs each. Global loads are coalesced along whichever dimension of A / B is contiguous (A_KC: A's K is
// contiguous, else its M; B_KC: B's K is contiguous, else its N); the next K-slab is fetched into registers while the
// current one is multiplied. grid.z splits K into chunks written to separate slabs (reduced in a fixed order).
template <typename TA, typename TB, bool A_KC, bool B_KC>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const TA* __restrict__ A, int64_t sam, int64_t sak,
                                                        const TB* __restrict__ B, int64_t sbk, int64_t sbn,
                                                        float* __restrict__ C, int64_t ldc, int M, int N, int K,
                                                        int k_chunk, float alpha, int accumulate) {
  constexpr int BM = 64, BN = 64, BK = 32;
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int kbeg = blockIdx.z * k_chunk;
  const int kend = min(K, kbeg + k_chunk);
  float ra[8], rb[8];  // 64*32 / 256 = 8 elements of each tile per thread
  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i;
      const int mm = A_KC ? idx / BK : idx % BM;
      const int ka = A_KC ? idx % BK : idx / BM;
      const int gm = m0 + mm, gk = k0 + ka;
      ra[i] = (gm < M && gk < kend) ? to_float(A[gm * sam + gk * sak]) : 0.f;
      const int nn = B_KC ? idx / BK : idx % BN;
      const int kb = B_KC ? idx % BK : idx / BN;
      const int gn = n0 + nn, gkb = k0 + kb;
      rb[i] = (gn < N && gkb < kend) ? to_float(B[gkb * sbk + gn * sbn]) : 0.f;
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i;
      As[A_KC ? idx % BK : idx / BM][A_KC ? idx / BK : idx % BM] = ra[i];
      Bs[B_KC ? idx % BK : idx / BN][B_KC ? idx / BK : idx % BN] = rb[i];
    }
  };
  float acc[4][4] = {};
  if (kbeg < kend) fetch(kbeg);
  for (int k0 = kbeg; k0 < kend; k0 += BK) {
    __syncthreads();
    stash();
    __syncthreads();
    if (k0 + BK < kend) fetch(k0 + BK);  // next slab in flight during the math
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
  }
  float* Cz = C + static_cast<int64_t>(blockIdx.z) * M * ldc;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      const float v = alpha * acc[i][j];
      Cz[static_cast<int64_t>(gm) * ldc + gn] = accumulate ? Cz[static_cast<int64_t>(gm) * ldc + gn] + v : v;
    }
  }
}

// out[i] (+)= sum_z part[z*n + i]  (fixed order)
__global__ void slab_sum_kernel(const float* __restrict__ part, int slabs, int64_t n, float* __restrict__ out,
                                int accumulate) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int z = 0; z < slabs; ++z) s += part[z * n + i];
  out[i] = accumulate ? out[i] + s : s;
}

// ------------------------------------------------------------------------------------------------ softmax + top-k
template <int EPL>
__global__ void router_topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int64_t T, int E,
                                   int k, float inv_temp_div, float temperature, float* __restrict__ probs,
                                   int* __restrict__ top_idx, float* __restrict__ top_w, int* __restrict__ counts) {
  const int warps = blockDim.x / 32;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float l[EPL], p[EPL], key[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    l[i] = (e < E) ? logits[t * E + e] / temperature : -INFINITY;
    mx = fmaxf(mx, l[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    p[i] = (e < E) ? __expf(l[i] - mx) : 0.f;
    sum += p[i];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    p[i] *= inv;
    if (e < E) probs[t * E + e] = p[i];
    key[i] = (e < E) ? (bias ? l[i] + bias[e] : p[i]) : -INFINITY;
  }
  float wsel[8];
  int isel[8];
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (key[i] > best || (key[i] == best && e < best_e))) { best = key[i]; best_e = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) { best = ob; best_e = oe; }
    }
    // the owner lane retires the chosen expert and broadcasts its probability
    float chosen_p = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i == best_e) { chosen_p = p[i]; key[i] = -INFINITY; }
    chosen_p = __shfl_sync(0xffffffffu, chosen_p, best_e % 32);
    isel[j] = best_e;
    wsel[j] = chosen_p;
    wsum += chosen_p;
  }
  if (lane < k) {
    float w = 0.f;
    int e = 0;
    for (int j = 0; j < k; ++j)
      if (j == lane) { w = wsel[j]; e = isel[j]; }
    top_idx[t * k + lane] = e;
    top_w[t * k + lane] = w / wsum;
    atomicAdd(&counts[e], 1);
  }
  (void)inv_temp_div;
}

// ------------------------------------------------------------------------------------------------ plan
// One block: kept = min(count, cap); padded offsets; unpadded offsets; meta = {total padded rows, overflow}
// slot_rows > 0: fixed slots (expert e starts at e * slot_rows) for even expert-parallel exchanges.
__global__ void plan_kernel(const int* __restrict__ counts, int E, int cap, int slot_rows, int* __restrict__ kept,
                            int* __restrict__ offsets, int* __restrict__ uoffsets, int* __restrict__ meta) {
  __shared__ int s_pad[1024];
  __shared__ int s_cnt[1024];
  __shared__ int s_over[1024];
  const int e = threadIdx.x;
  const int c = e < E ? counts[e] : 0;
  const int kc = min(c, cap);
  s_pad[e] = e < E ? ((kc + 127) / 128) * 128 : 0;
  s_cnt[e] = c;
  s_over[e] = c - kc;
  __syncthreads();
  if (e == 0) {
    int acc = 0, uacc = 0, over = 0;
    for (int i = 0; i < E; ++i) {
      const int pad = s_pad[i];
      s_pad[i] = acc;
      acc += pad;
      const int cnt = s_cnt[i];
      s_cnt[i] = uacc;
      uacc += cnt;
      over += s_over[i];
    }
    meta[0] = slot_rows > 0 ? E * slot_rows : acc;
    meta[1] = over;
  }
  __syncthreads();
  if (e < E) {
    kept[e] = kc;
    offsets[e] = slot_rows > 0 ? e * slot_rows : s_pad[e];
    uoffsets[e] = s_cnt[e];
  }
}

// ------------------------------------------------------------------------------------------------ stable rank
constexpr int kChunk = 2048;

__global__ void chunk_hist_kernel(const int* __restrict__ top_idx, int64_t routes, int E, int* __restrict__ hist) {
  extern __shared__ int sh[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kChunk;
  for (int i = threadIdx.x; i < kChunk; i += blockDim.x) {
    const int64_t r = base + i;
    if (r < routes) atomicAdd(&sh[top_idx[r]], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[static_cast<int64_t>(blockIdx.x) * E + e] = sh[e];
}

// hist[c][e] -> exclusive prefix over chunks (in place)
__global__ void chunk_scan_kernel(int* __restrict__ hist, int chunks, int E) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  int acc = 0;
  for (int c = 0; c < chunks; ++c) {
    const int v = hist[static_cast<int64_t>(c) * E + e];
    hist[static_cast<int64_t>(c) * E + e] = acc;
    acc += v;
  }
}

// 1024 threads, E <= 512: stable rank of each route within its expert.
__global__ void __launch_bounds__(1024) rank_kernel(const int* __restrict__ top_idx, int64_t routes, int E, int cap,
                                                    const int* __restrict__ chunk_base, const int* __restrict__ counts,
                                                    const int* __restrict__ offsets, const int* __restrict__ uoffsets,
                                                    int* __restrict__ sorted_routes, int* __restrict__ route_row) {
  extern __shared__ int sh[];
  int* wcount = sh;            // [32][E]
  int* running = sh + 32 * E;  // [E]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int i = threadIdx.x; i < 33 * E; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kChunk;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int pass = 0; pass < kChunk / 1024; ++pass) {
    const int64_t r = base + pass * 1024 + threadIdx.x;
    const bool valid = r < routes;
    const int e = valid ? top_idx[r] : -1 - lane;  // invalid lanes never match anyone
    const unsigned mask = __match_any_sync(0xffffffffu, e);
    const int lane_rank = __popc(mask & lt_mask);
    if (valid && lane_rank == 0) wcount[warp * E + e] = __popc(mask);
    __syncthreads();
    if (valid) {
      int rank = running[e] + lane_rank;
      for (int w = 0; w < warp; ++w) rank += wcount[w * E + e];
      rank += chunk_base[static_cast<int64_t>(blockIdx.x) * E + e];
      sorted_routes[uoffsets[e] + rank] = static_cast<int>(r);
      route_row[r] = (counts[e] <= cap) ? offsets[e] + rank : -2;
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
      int s = 0;
      for (int w = 0; w < 32; ++w) {
        s += wcount[w * E + ee];
        wcount[w * E + ee] = 0;
      }
      running[ee] += s;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------ select
__device__ __forceinline__ uint64_t route_key(float w, int route) {
  uint32_t b = __float_as_uint(w);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving float -> unsigned
  return (static_cast<uint64_t>(b) << 32) | static_cast<uint32_t>(0xFFFFFFFFu - static_cast<uint32_t>(route));
}

// One block per expert; only experts over capacity do work. Keeps the `cap` largest keys, in route order.
__global__ void __launch_bounds__(1024) select_kernel(const int* __restrict__ counts, int cap,
                                                      const int* __restrict__ offsets,
                                                      const int* __restrict__ uoffsets,
                                                      const int* __restrict__ sorted_routes,
                                                      const float* __restrict__ top_w, int* __restrict__ route_row) {
  const int e = blockIdx.x;
  const int n = counts[e];
  if (n <= cap) return;
  __shared__ int hist[256];
  __shared__ uint64_t s_prefix;
  __shared__ int s_need;
  __shared__ int s_scan[1024];
  __shared__ int s_carry;
  const int* seg = sorted_routes + uoffsets[e];
  // The keys of one expert share their leading bytes (route weights of similar size): the bytes above the first
  // one in which two keys differ take no radix pass. These passes were the slowest, every key landing in one bin.
  __shared__ unsigned long long s_diff;
  if (threadIdx.x == 0) s_diff = 0;
  __syncthreads();
  const uint64_t key0 = route_key(top_w[seg[0]], seg[0]);
  uint64_t diff = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) diff |= route_key(top_w[seg[i]], seg[i]) ^ key0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) diff |= __shfl_xor_sync(0xffffffffu, diff, o);
  if ((threadIdx.x & 31) == 0 && diff) atomicOr(&s_diff, static_cast<unsigned long long>(diff));
  __syncthreads();
  const uint64_t differ = s_diff;
  const int first_shift = differ ? ((63 - __clzll(static_cast<long long>(differ))) / 8) * 8 : 0;
  if (threadIdx.x == 0) {  // rank (1-based) of the threshold among the largest keys; the shared leading bytes
    s_need = cap;
    s_prefix = first_shift == 56 ? 0ull : (key0 & (~0ull << (first_shift + 8)));
  }
  __syncthreads();
  for (int shift = first_shift; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint64_t prefix = s_prefix;
    const uint64_t hi_mask = (shift == 56) ? 0ull : (~0ull << (shift + 8));
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int r = seg[i];
      const uint64_t key = route_key(top_w[r], r);
      if ((key & hi_mask) == (prefix & hi_mask)) atomicAdd(&hist[(key >> shift) & 0xFF], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int need = s_need;
      int digit = 255;
      for (; digit > 0; --digit) {
        if (hist[digit] >= need) break;
        need -= hist[digit];
      }
      s_need = need;
      s_prefix = prefix | (static_cast<uint64_t>(digit) << shift);
    }
    __syncthreads();
  }
  const uint64_t threshold = s_prefix;  // exactly `cap` keys are >= threshold (keys are unique)
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int keep = 0, r = 0;
    if (i < n) {
      r = seg[i];
      keep = route_key(top_w[r], r) >= threshold;
    }
    s_scan[threadIdx.x] = keep;
    __syncthreads();
    for (int off = 1; off < blockDim.x; off <<= 1) {  // inclusive Hillis-Steele scan
      const int v = threadIdx.x >= off ? s_scan[threadIdx.x - off] : 0;
      __syncthreads();
      s_scan[threadIdx.x] += v;
      __syncthreads();
    }
    if (i < n) route_row[r] = keep ? offsets[e] + s_carry + s_scan[threadIdx.x] - 1 : -1;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) s_carry += s_scan[threadIdx.x];
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------ permute
// one warp per route; x_perm[row] = x[token]
__global__ void permute_kernel(const bf16* __restrict__ x, int64_t routes, int k, int H,
                               const int* __restrict__ route_row, const float* __restrict__ top_w,
                               bf16* __restrict__ x_perm, int* __restrict__ row_token, float* __restrict__ row_w,
                               int64_t perm_rows) {
  const int warps = blockDim.x / 32;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (r >= routes) return;
  const int row = route_row[r];
  if (row < 0 || !in_bounds(row, perm_rows)) return;
  const int64_t t = r / k;
  if (lane == 0) {
    row_token[row] = static_cast<int>(t);
    row_w[row] = top_w[r];
  }
  const uint4* src = reinterpret_cast<const uint4*>(x + t * H);
  uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<int64_t>(row) * H);
  for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
}

// zero the padding rows of every expert segment: block per (expert, 128-row chunk)
__global__ void pad_rows_kernel(const int* __restrict__ kept, const int* __restrict__ offsets, int H,
                                bf16* __restrict__ x_perm, int* __restrict__ row_token, float* __restrict__ row_w) {
  const int e = blockIdx.x;
  const int n = kept[e];
  const int pad_end = ((n + 127) / 128) * 128;
  const int64_t first = offsets[e];
  for (int row = n + threadIdx.y; row < pad_end; row += blockDim.y) {
    const int64_t gr = first + row;
    if (threadIdx.x == 0) {
      if (row_token) row_token[gr] = -1;
      if (row_w) row_w[gr] = 0.f;
    }
    if (x_perm) {
      uint4* dst = reinterpret_cast<uint4*>(x_perm + gr * H);
      for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    }
  }
}

// dst[row] = src[row_token[row]] (zero for padding rows), rows < meta[0]
__global__ void gather_rows_kernel(const bf16* __restrict__ src, const int* __restrict__ row_token,
                                   const int* __restrict__ meta, int64_t max_rows, int H, bf16* __restrict__ dst) {
  const int warps = blockDim.x / 32;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= max_rows || row >= meta[0]) return;
  const int t = row_token[row];
  uint4* d = reinterpret_cast<uint4*>(dst + row * H);
  if (t < 0) {
    for (int c = lane; c < H / 8; c += 32) d[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(t) * H);
  for (int c = lane; c < H / 8; c += 32) d[c] = s[c];
}

// ------------------------------------------------------------------------------------------------ combine
// out[t] = resid[t] + sum_j w_j * y[row(t,j)] ; one warp per token, 8 columns per lane step
__global__ void combine_kernel(const bf16* __restrict__ y, const int* __restrict__ route_row,
                               const float* __restrict__ top_w, const bf16* __restrict__ resid, int64_t T, int k, int H,
                               bf16* __restrict__ out, int64_t y_rows) {
  const int warps = blockDim.x / 32;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  int rows[8];
  float ws[8];
  for (int j = 0; j < k; ++j) {
    rows[j] = route_row[t * k + j];
    ws[j] = top_w[t * k + j];
  }
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {};
    for (int j = 0; j < k; ++j) {
      if (rows[j] < 0 || !in_bounds(rows[j], y_rows)) continue;
      uint4 raw = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(rows[j]) * H + c);
      const bf16* v = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += ws[j] * __bfloat162float(v[i]);
    }
    if (resid) {
      uint4 raw = *reinterpret_cast<const uint4*>(resid + t * H + c);
      const bf16* v = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __bfloat162float(v[i]) + __bfloat162float(__float2bfloat16(acc[i]));
    }
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]); o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]); o.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + t * H + c) = o;
  }
}

// dx[t] = extra[t] (fp32, optional) + sum_j dx_perm[row(t,j)]   (unweighted: the route weight was applied upstream)
__global__ void combine_grad_kernel(const bf16* __restrict__ dx_perm, const int* __restrict__ route_row,
                                    const float* __restrict__ extra, int64_t T, int k, int H, bf16* __restrict__ dx,
                                    int64_t perm_rows) {
  const int warps = blockDim.x / 32;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  int rows[8];
  for (int j = 0; j < k; ++j) rows[j] = route_row[t * k + j];
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {};
    if (extra) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = extra[t * H + c + i];
    }
    for (int j = 0; j < k; ++j) {
      if (rows[j] < 0 || !in_bounds(rows[j], perm_rows)) continue;
      uint4 raw = *reinterpret_cast<const uint4*>(dx_perm + static_cast<int64_t>(rows[j]) * H + c);
      const bf16* v = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(v[i]);
    }
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]); o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]); o.w = pack_bf16(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(dx + t * H + c) = o;
  }
}

// d_w[route] = sum_tiles partial[row, tile]  (0 for dropped routes)
__global__ void route_dw_kernel(const float* __restrict__ partial, int tiles, const int* __restrict__ route_row,
                                int64_t routes, float* __restrict__ d_w) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= routes) return;
  const int row = route_row[r];
  float s = 0.f;
  if (row >= 0)
    for (int i = 0; i < tiles; ++i) s += partial[static_cast<int64_t>(row) * tiles + i];
  d_w[r] = s;
}

// softmax + renormalisation backward: d_logits[t,e] (already divided by the temperature)
template <int EPL>
__global__ void router_bwd_kernel(const float* __restrict__ probs, const int* __restrict__ top_idx,
                                  const float* __restrict__ top_w, const float* __restrict__ d_w,
                                  const float* __restrict__ d_probs_ext, int64_t T, int E, int k, float temperature,
                                  float* __restrict__ d_logits) {
  const int warps = blockDim.x / 32;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  // renormalised weights w_j = p_j / S:  dp_j = (dw_j - sum_i dw_i w_i) / S
  float dot = 0.f, S = 0.f;
  for (int j = 0; j < k; ++j) {
    dot += d_w[t * k + j] * top_w[t * k + j];
    S += probs[t * E + top_idx[t * k + j]];
  }
  float p[EPL], dp[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? probs[t * E + e] : 0.f;
    dp[i] = (e < E && d_probs_ext) ? d_probs_ext[t * E + e] : 0.f;
  }
  for (int j = 0; j < k; ++j) {
    const int e = top_idx[t * k + j];
    if (e % 32 == lane) {
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (lane + 32 * i == e) dp[i] += (d_w[t * k + j] - dot) / S;
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) s += p[i] * dp[i];
  s = warp_sum(s);
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) d_logits[t * E + e] = p[i] * (dp[i] - s) / temperature;
  }
}

template <typename TA, typename TB, bool AK, bool BK>
void launch_simt(dim3 grid, const TA* A, int64_t sam, int64_t sak, const TB* B, int64_t sbk, int64_t sbn, float* C,
                 int64_t ldc, int M, int N, int K, int k_chunk, float alpha, int accumulate, cudaStream_t stream) {
  simt_gemm_kernel<TA, TB, AK, BK><<<grid, 256, 0, stream>>>(A, sam, sak, B, sbk, sbn, C, ldc, M, N, K, k_chunk, alpha,
                                                             accumulate);
}

template <typename TA, typename TB>
void simt_gemm(const TA* A, int64_t sam, int64_t sak, const TB* B, int64_t sbk, int64_t sbn, float* C, int64_t ldc,
               int M, int N, int K, float alpha, bool accumulate, float* workspace, int split_k, cudaStream_t stream) {
  if (M == 0 || N == 0) return;
  split_k = std::max(1, std::min(split_k, (K + 31) / 32));
  const int k_chunk = ((K + split_k - 1) / split_k + 31) / 32 * 32;
  split_k = std::max(1, (K + k_chunk - 1) / k_chunk);
  dim3 grid((N + 63) / 64, (M + 63) / 64, split_k);
  const bool ak = sak == 1, bk = sbk == 1;  // which dimension of each operand is contiguous
  float* out = split_k == 1 ? C : workspace;
  const int64_t ld = split_k == 1 ? ldc : N;
  const int acc = split_k == 1 && accumulate ? 1 : 0;
  if (ak && bk) launch_simt<TA, TB, true, true>(grid, A, sam, sak, B, sbk, sbn, out, ld, M, N, K, k_chunk, alpha, acc, stream);
  else if (ak) launch_simt<TA, TB, true, false>(grid, A, sam, sak, B, sbk, sbn, out, ld, M, N, K, k_chunk, alpha, acc, stream);
  else if (bk) launch_simt<TA, TB, false, true>(grid, A, sam, sak, B, sbk, sbn, out, ld, M, N, K, k_chunk, alpha, acc, stream);
  else launch_simt<TA, TB, false, false>(grid, A, sam, sak, B, sbk, sbn, out, ld, M, N, K, k_chunk, alpha, acc, stream);
  if (split_k > 1) {
    const int64_t n = static_cast<int64_t>(M) * N;
    slab_sum_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, stream>>>(workspace, split_k, n, C, accumulate);
  }
  check_cuda(cudaGetLastError(), "simt_gemm");
}

}  // namespace

// ================================================================================================ launchers
void router_logits(const bf16* x, const float* w, int64_t T, int H, int E, float* logits, cudaStream_t stream) {
  simt_gemm<bf16, float>(x, H, 1, w, 1, H, logits, E, static_cast<int>(T), E, H, 1.f, false, nullptr, 1, stream);
}

void router_topk(const float* logits, const float* bias, int64_t T, int E, int k, float temperature, float* probs,
                 int* top_idx, float* top_w, int* counts, cudaStream_t stream) {
  if (k > 8 || k > E) throw std::runtime_error("router: top_k must be <= min(8, experts)");
  check_cuda(cudaMemsetAsync(counts, 0, E * sizeof(int), stream), "counts memset");
  if (T == 0) return;
  const int warps = 8;
  const int grid = static_cast<int>((T + warps - 1) / warps);
  const int epl = (E + 31) / 32;
#define QW_TOPK(N) router_topk_kernel<N><<<grid, warps * 32, 0, stream>>>(logits, bias, T, E, k, 0.f, temperature, \
                                                                          probs, top_idx, top_w, counts)
  if (epl <= 1) QW_TOPK(1);
  else if (epl <= 2) QW_TOPK(2);
  else if (epl <= 4) QW_TOPK(4);
  else if (epl <= 8) QW_TOPK(8);
  else if (epl <= 32) QW_TOPK(32);
  else throw std::runtime_error("router: at most 1024 experts");
#undef QW_TOPK
  check_cuda(cudaGetLastError(), "router_topk");
}

int moe_plan_chunks(int64_t routes) { return static_cast<int>((routes + kChunk - 1) / kChunk); }

void moe_plan(const int* top_idx, const float* top_w, const int* counts, int64_t routes, int E, int cap, int slot_rows,
              int* kept, int* offsets, int* uoffsets, int* meta, int* chunk_hist, int* sorted_routes, int* route_row,
              cudaStream_t stream) {
  if (E > 512) throw std::runtime_error("moe_plan: at most 512 experts");
  if (slot_rows > 0 && (slot_rows % 128 || slot_rows < cap))
    throw std::runtime_error("moe_plan: slot rows must be a multiple of 128 that holds the capacity");
  plan_kernel<<<1, 1024, 0, stream>>>(counts, E, cap, slot_rows, kept, offsets, uoffsets, meta);
  const int chunks = moe_plan_chunks(routes);
  if (chunks > 0) {
    chunk_hist_kernel<<<chunks, 256, E * sizeof(int), stream>>>(top_idx, routes, E, chunk_hist);
    chunk_scan_kernel<<<(E + 255) / 256, 256, 0, stream>>>(chunk_hist, chunks, E);
    const size_t smem = 33 * E * sizeof(int);
    check_cuda(cudaFuncSetAttribute(rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "rank smem");
    rank_kernel<<<chunks, 1024, smem, stream>>>(top_idx, routes, E, cap, chunk_hist, counts, offsets, uoffsets,
                                                sorted_routes, route_row);
    select_kernel<<<E, 1024, 0, stream>>>(counts, cap, offsets, uoffsets, sorted_routes, top_w, route_row);
  }
  check_cuda(cudaGetLastError(), "moe_plan");
}

void moe_permute(const bf16* x, int64_t routes, int k, int H, const int* route_row, const float* top_w, const int* kept,
                 const int* offsets, int E, bf16* x_perm, int* row_token, float* row_w, int64_t perm_rows,
                 cudaStream_t stream) {
  if (H % 8) throw std::runtime_error("moe_permute: hidden size must be a multiple of 8");
  if (routes > 0) {
    const int warps = 8;
    permute_kernel<<<static_cast<int>((routes + warps - 1) / warps), warps * 32, 0, stream>>>(
        x, routes, k, H, route_row, top_w, x_perm, row_token, row_w, perm_rows);
  }
  pad_rows_kernel<<<E, dim3(32, 8), 0, stream>>>(kept, offsets, H, x_perm, row_token, row_w);
  check_cuda(cudaGetLastError(), "moe_permute");
}

void moe_pad_zero(const int* kept, const int* offsets, int E, int H, bf16* buf, cudaStream_t stream) {
  pad_rows_kernel<<<E, dim3(32, 8), 0, stream>>>(kept, offsets, H, buf, nullptr, nullptr);
  check_cuda(cudaGetLastError(), "moe_pad_zero");
}

void moe_gather_rows(const bf16* src, const int* row_token, const int* meta, int64_t max_rows, int H, bf16* dst,
                     cudaStream_t stream) {
  if (max_rows == 0) return;
  const int warps = 8;
  gather_rows_kernel<<<static_cast<int>((max_rows + warps - 1) / warps), warps * 32, 0, stream>>>(src, row_token, meta,
                                                                                                  max_rows, H, dst);
  check_cuda(cudaGetLastError(), "moe_gather_rows");
}

void moe_combine(const bf16* y, const int* route_row, const float* top_w, const bf16* resid, int64_t T, int k, int H,
                 bf16* out, int64_t y_rows, cudaStream_t stream) {
  if (T == 0) return;
  if (k > 8) throw std::runtime_error("moe_combine: top_k must be <= 8");
  const int warps = 8;
  combine_kernel<<<static_cast<int>((T + warps - 1) / warps), warps * 32, 0, stream>>>(y, route_row, top_w, resid, T, k,
                                                                                       H, out, y_rows);
  check_cuda(cudaGetLastError(), "moe_combine");
}

void moe_combine_grad(const bf16* dx_perm, const int* route_row, const float* extra, int64_t T, int k, int H, bf16* dx,
                      int64_t perm_rows, cudaStream_t stream) {
  if (T == 0) return;
  if (k > 8) throw std::runtime_error("moe_combine_grad: top_k must be <= 8");
  const int warps = 8;
  combine_grad_kernel<<<static_cast<int>((T + warps - 1) / warps), warps * 32, 0, stream>>>(dx_perm, route_row, extra,
                                                                                            T, k, H, dx, perm_rows);
  check_cuda(cudaGetLastError(), "moe_combine_grad");
}

void moe_route_dw(const float* partial, int tiles, const int* route_row, int64_t routes, float* d_w,
                  cudaStream_t stream) {
  if (routes == 0) return;
  route_dw_kernel<<<static_cast<int>((routes + 255) / 256), 256, 0, stream>>>(partial, tiles, route_row, routes, d_w);
  check_cuda(cudaGetLastError(), "moe_route_dw");
}

void router_backward(const float* probs, const int* top_idx, const float* top_w, const float* d_w,
                     const float* d_probs_ext, int64_t T, int E, int k, float temperature, float* d_logits,
                     cudaStream_t stream) {
  if (T == 0) return;
  const int warps = 8;
  const int grid = static_cast<int>((T + warps - 1) / warps);
  const int epl = (E + 31) / 32;
#define QW_RB(N) router_bwd_kernel<N><<<grid, warps * 32, 0, stream>>>(probs, top_idx, top_w, d_w, d_probs_ext, T, E, k, \
                                                                       temperature, d_logits)
  if (epl <= 1) QW_RB(1);
  else if (epl <= 2) QW_RB(2);
  else if (epl <= 4) QW_RB(4);
  else if (epl <= 8) QW_RB(8);
  else QW_RB(32);
#undef QW_RB
  check_cuda(cudaGetLastError(), "router_backward");
}

// dx_router[T,H] = d_logits[T,E] . Wr[E,H]   (fp32 out)
void router_dx(const float* d_logits, const float* w, int64_t T, int E, int H, float* dx, cudaStream_t stream) {
  simt_gemm<float, float>(d_logits, E, 1, w, H, 1, dx, H, static_cast<int>(T), H, E, 1.f, false, nullptr, 1, stream);
}

// dWr[E,H] (+)= d_logits^T . x    (split-K over tokens, fixed-order reduction); workspace >= split*E*H floats
int router_dw_split(int64_t T) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(64, T / 1024))); }

void router_dw(const float* d_logits, const bf16* x, int64_t T, int E, int H, float* dw, bool accumulate,
               float* workspace, cudaStream_t stream) {
  simt_gemm<float, bf16>(d_logits, 1, E, x, H, 1, dw, H, E, H, static_cast<int>(T), 1.f, accumulate, workspace,
                         router_dw_split(T), stream);
}

// ------------------------------------------------------------------------------------------------ router GEMMs on
// the tensor cores. An fp32 operand is split into bf16 parts (a = hi + mid + lo to ~24 mantissa bits, or hi + lo to
// ~16); a bf16 x bf16 product is exact in fp32, so the tcgen05 GEMM over the stacked parts reproduces the fp32 GEMM
// up to summation order. The MoE input x is bf16 already and needs no split.
namespace {

__global__ void split_w_kernel(const float* __restrict__ w, int64_t n, bf16* __restrict__ out, int mode) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = w[i];
    const bf16 hi = __float2bfloat16(a);
    const float r = a - __bfloat162float(hi);
    const bf16 mid = __float2bfloat16(r);
    const bf16 lo = __float2bfloat16(r - __bfloat162float(mid));
    out[i] = hi;
    out[n + i] = mode == 0 ? mid : hi;   // mode 0: [hi; mid; lo]   mode 1: [hi; hi; mid] (two-term split twice)
    out[2 * n + i] = mode == 0 ? lo : mid;
  }
}

// d[T,E] -> out[T,3E] = [hi | lo | hi]
__global__ void split_dl_kernel(const float* __restrict__ d, int64_t total, int E, bf16* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / E;
    const int e = static_cast<int>(i % E);
    const float a = d[i];
    const bf16 hi = __float2bfloat16(a);
    const bf16 lo = __float2bfloat16(a - __bfloat162float(hi));
    bf16* row = out + t * 3 * E;
    row[e] = hi;
    row[E + e] = lo;
    row[2 * E + e] = hi;
  }
}

// logits[t,e] = part_hi + (part_mid + part_lo)
__global__ void sum3_kernel(const float* __restrict__ in, int64_t total, int E, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / E;
    const int e = static_cast<int>(i % E);
    const float* row = in + t * 3 * E;
    out[i] = row[e] + (row[E + e] + row[2 * E + e]);
  }
}

// dw[e,h] (+)= sum over chunks c in order of (partial[c][e][h] + partial[c][E+e][h])
__global__ void dw_reduce_kernel(const float* __restrict__ partial, int chunks, int64_t eh, float* __restrict__ dw,
                                 bool accumulate) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < eh;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = 0.f;
    for (int c = 0; c < chunks; ++c) acc += partial[c * 2 * eh + i] + partial[c * 2 * eh + eh + i];
    dw[i] = accumulate ? dw[i] + acc : acc;
  }
}

int elementwise_grid(int64_t n) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(4096, (n + 255) / 256))); }

}  // namespace

bool router_tc_ok(int64_t T, int H, int E) { return T >= 256 && H % 64 == 0 && E % 8 == 0; }

void router_logits_tc(const bf16* x, const float* w, int64_t T, int H, int E, float* logits, bf16* w3, float* out3,
                      cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(E) * H;
  split_w_kernel<<<elementwise_grid(n), 256, 0, stream>>>(w, n, w3, 0);
  linear_fwd(x, H, w3, H, T, 3 * E, H, nullptr, nullptr, 0, out3, 3 * E, true, stream);
  sum3_kernel<<<elementwise_grid(T * E), 256, 0, stream>>>(out3, T * E, E, logits);
  check_cuda(cudaGetLastError(), "router_logits_tc");
}

void router_dx_tc(const float* d_logits, const float* w, int64_t T, int E, int H, float* dx, bf16* dls, bf16* w3,
                  cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(E) * H;
  split_dl_kernel<<<elementwise_grid(T * E), 256, 0, stream>>>(d_logits, T * E, E, dls);
  split_w_kernel<<<elementwise_grid(n), 256, 0, stream>>>(w, n, w3, 1);
  // dx = [dl_hi | dl_lo | dl_hi] . [W_hi; W_hi; W_lo]
  linear_dgrad(dls, 3 * E, w3, H, T, 3 * E, H, dx, H, true, false, stream);
  check_cuda(cudaGetLastError(), "router_dx_tc");
}

int64_t router_dw_chunk(int64_t T, int H) {
  // enough chunks that chunks x (H / 256) output tiles cover the 148 SMs about once
  const int64_t tiles = std::max<int64_t>(1, (H + 255) / 256);
  const int64_t chunks = std::max<int64_t>(1, 148 / tiles);
  const int64_t chunk = (T + chunks - 1) / chunks;
  return std::max<int64_t>(64, (chunk + 63) / 64 * 64);
}

void router_dw_tc(const float* d_logits, const bf16* x, int64_t T, int E, int H, float* dw, bool accumulate,
                  bf16* dls, float* partial, cudaStream_t stream) {
  split_dl_kernel<<<elementwise_grid(T * E), 256, 0, stream>>>(d_logits, T * E, E, dls);
  const int64_t chunk = router_dw_chunk(T, H);
  const int chunks = static_cast<int>((T + chunk - 1) / chunk);
  // partial[c] = [dl_hi | dl_lo]^T . x over the chunk's tokens: 2E x H
  linear_wgrad_chunks(dls, 3 * E, x, H, T, 2 * E, H, chunk, partial, stream);
  const int64_t eh = static_cast<int64_t>(E) * H;
  dw_reduce_kernel<<<elementwise_grid(eh), 256, 0, stream>>>(partial, chunks, eh, dw, accumulate);
  check_cuda(cudaGetLastError(), "router_dw_tc");
}

int routing_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
