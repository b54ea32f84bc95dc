// Decode-time kernels (one new token per sequence, small batch, memory/latency bound). Every kernel is launched with
// programmatic dependent launch: it may be scheduled while the previous kernel drains, prefetches what does not
// depend on it (weights), then waits on `griddepcontrol.wait` before touching activations.
//
//  * grouped GEMV over weight formats bf16 / int8 (one fp16 scale per row) / int4 (fp16 scale per group of columns,
//    two values per byte, low nibble = even column, stored +8): out[r, n] = sum_k x[tok(r), k] * W[g(r)][n, k].
//    A warp owns two output rows of one group (expert), issues all of its weight loads before the math, and keeps
//    four routed tokens in flight per pass. No shared memory, so every block of a decode GEMV is resident at once.
//    The SwiGLU variant computes gate row n and up row n + N together and writes silu(gate) * up.
//  * split-K decode attention over a [B, Hkv, Lmax, D] bf16 KV cache: one block per (64-key chunk, batch x kv head)
//    serves every q head of that kv head; D/8 lanes share a key so a warp issues its 16 key loads at once. The last
//    chunk block of a (batch, kv head) to finish merges the chunks by log-sum-exp (ticket counter, reset by it).
//  * routing: router logits (one block per expert), the last block does softmax / top-k / per-expert lists.
//  * combine + norm: residual + sum_j w_j y[slot_j] (the MoE output of the previous layer), then LayerNorm/RMSNorm.
//  * RoPE + KV-cache append for the new token.
#include <algorithm>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* what,
                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

__device__ __forceinline__ void bf16x8_to_float(const uint4& raw, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// ------------------------------------------------------------------------------------------------ grouped GEMV
constexpr int kGemvWarps = 4;
constexpr int kGemvRows = 2;  // output rows per warp
constexpr int kGemvTok = 4;   // routed tokens per pass over the warp's weight rows

// A lane covers kVals consecutive columns of a row with one 16-byte weight load.
template <int FMT>
struct WF;

template <>
struct WF<0> {  // bf16
  static constexpr int kVals = 8;
  __device__ static int64_t byte_off(int k) { return static_cast<int64_t>(k) * 2; }
  __device__ static float dot(const uint4& raw, const float* x) {
    float w[8];
    bf16x8_to_float(raw, w);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += w[i] * x[i];
    return s;
  }
  __host__ __device__ static int64_t row_bytes(int K) { return static_cast<int64_t>(K) * 2; }
};

template <>
struct WF<1> {  // int8, one scale per row
  static constexpr int kVals = 16;
  __device__ static int64_t byte_off(int k) { return k; }
  __device__ static float dot(const uint4& raw, const float* x) {
    const int8_t* q = reinterpret_cast<const int8_t*>(&raw);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) s += static_cast<float>(q[i]) * x[i];
    return s;
  }
  __host__ __device__ static int64_t row_bytes(int K) { return K; }
};

template <>
struct WF<2> {  // int4 packed (+8), per-group scales, group a multiple of 32
  static constexpr int kVals = 32;
  __device__ static int64_t byte_off(int k) { return k / 2; }
  __device__ static float dot(const uint4& raw, const float* x) {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(&raw);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) s += static_cast<float>(static_cast<int>((q[i] >> (4 * j)) & 0xFu) - 8) * x[8 * i + j];
    return s;
  }
  __host__ __device__ static int64_t row_bytes(int K) { return K / 2; }
};

struct GemvArgs {
  const bf16* x;
  int64_t ldx;
  const uint8_t* w;
  const __half* s;
  int64_t wgb;  // bytes per group (expert) of w
  int64_t sge;  // scales per group
  int N, K, group;
  const int* tok;     // routed entry -> row of x (nullptr: identity)
  const int* off;     // per-group first entry (nullptr: 0)
  const int* cnt;     // per-group entries (nullptr: dense_rows)
  int dense_rows;
  bf16* out;
  int64_t ldo;
  int out_by_route;   // output row = entry index (else the token row)
  const float* bias;  // [N] or nullptr
  const bf16* resid;  // added in the epilogue, same row as out
  int64_t ldr;
  const int* active;  // compact list of groups with entries (-1 padded); nullptr: blockIdx.y is the group
};

template <int FMT, bool SWIGLU, bool PRE>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const GemvArgs a) {
  using F = WF<FMT>;
  constexpr int NW = SWIGLU ? 2 * kGemvRows : kGemvRows;  // weight rows per warp
  constexpr int KU = (FMT == 0 ? 4 : 2) / (SWIGLU ? 2 : 1);  // k steps whose loads are issued together
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n0 = (blockIdx.x * kGemvWarps + warp) * kGemvRows;
  const int64_t rb = F::row_bytes(a.K);
  const bool routed = a.active != nullptr || a.cnt != nullptr;
  const int spr = (FMT == 2) ? a.K / a.group : 1;  // scales per row
  const uint8_t* wrow[NW];
  const __half* srow[NW];
  bool ok[NW];
  auto rows_of = [&](int g) {
#pragma unroll
    for (int r = 0; r < NW; ++r) {
      const int n = n0 + r % kGemvRows;
      ok[r] = n < a.N;
      const int64_t wn = ok[r] ? n + static_cast<int64_t>(r / kGemvRows) * a.N : 0;
      wrow[r] = a.w + static_cast<int64_t>(g) * a.wgb + wn * rb;
      srow[r] = a.s ? a.s + static_cast<int64_t>(g) * a.sge + wn * spr : nullptr;
    }
  };
  auto load = [&](int kb, uint4 (&wv)[KU][NW], float (&sc)[KU][NW]) {
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int k = kb + u * 32 * F::kVals;
#pragma unroll
      for (int r = 0; r < NW; ++r) {
        const bool live = ok[r] && k < a.K;
        wv[u][r] = live ? __ldg(reinterpret_cast<const uint4*>(wrow[r] + F::byte_off(k))) : make_uint4(0, 0, 0, 0);
        sc[u][r] = (FMT == 0 || !live) ? 1.f : __half2float(srow[r][FMT == 2 ? k / a.group : 0]);
      }
    }
  };
  // Dense rows (PRE: no routing lists) do not depend on the previous kernel: the first k-block of this warp's
  // weights is loaded into registers before the programmatic-launch wait (for a 1024-wide bf16 row that is the
  // whole row), the rest is pulled into L2. Routed launches keep those registers free.
  const bool pre = PRE && !routed && n0 < a.N;
  uint4 wpre[PRE ? KU : 1][NW];
  float spre[PRE ? KU : 1][NW];
  if constexpr (PRE) {
   if (pre) {
    rows_of(blockIdx.y);
    load(lane * F::kVals, wpre, spre);
#pragma unroll
    for (int r = 0; r < NW; ++r) {
      if (!ok[r]) continue;
      for (int64_t b = static_cast<int64_t>(lane) * 128 + KU * 32 * 16; b < rb; b += 32 * 128) prefetch_l2(wrow[r] + b);
    }
   }
  }
  griddep_wait();
  griddep_launch();
  const int g = a.active ? a.active[blockIdx.y] : blockIdx.y;
  if (g < 0 || n0 >= a.N) return;
  const int count = a.cnt ? a.cnt[g] : a.dense_rows;
  if (count <= 0) return;
  const int base = a.off ? a.off[g] : 0;
  if (!pre) rows_of(g);
  for (int c0 = 0; c0 < count; c0 += kGemvTok) {
    const int tc = min(kGemvTok, count - c0);
    const bf16* xr[kGemvTok];
#pragma unroll
    for (int t = 0; t < kGemvTok; ++t) {
      const int e = base + c0 + min(t, tc - 1);
      xr[t] = a.x + static_cast<int64_t>(a.tok ? a.tok[e] : e) * a.ldx;
    }
    float acc[NW][kGemvTok];
#pragma unroll
    for (int r = 0; r < NW; ++r)
#pragma unroll
      for (int t = 0; t < kGemvTok; ++t) acc[r][t] = 0.f;
    for (int kb = lane * F::kVals; kb < a.K; kb += KU * 32 * F::kVals) {
      uint4 wv[KU][NW];
      float sc[KU][NW];
      if constexpr (PRE) {
        if (pre && c0 == 0 && kb == lane * F::kVals) {
#pragma unroll
          for (int u = 0; u < KU; ++u)
#pragma unroll
            for (int r = 0; r < NW; ++r) { wv[u][r] = wpre[u][r]; sc[u][r] = spre[u][r]; }
        } else {
          load(kb, wv, sc);
        }
      } else {
        load(kb, wv, sc);
      }
#pragma unroll
      for (int u = 0; u < KU; ++u) {
        const int k = kb + u * 32 * F::kVals;
        if (k >= a.K) break;
#pragma unroll
        for (int t = 0; t < kGemvTok; ++t) {
          if (t < tc) {
            float xv[F::kVals];
#pragma unroll
            for (int i = 0; i < F::kVals; i += 8)
              bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(xr[t] + k + i)), xv + i);
#pragma unroll
            for (int r = 0; r < NW; ++r) acc[r][t] += sc[u][r] * F::dot(wv[u][r], xv);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kGemvTok; ++t)
      if (t < tc)
#pragma unroll
        for (int r = 0; r < NW; ++r) acc[r][t] = warp_sum(acc[r][t]);
#pragma unroll
    for (int ar = 0; ar < kGemvRows; ++ar)
#pragma unroll
      for (int t = 0; t < kGemvTok; ++t) {
        const int n = n0 + ar;
        if (lane == ar * kGemvTok + t && t < tc && n < a.N) {
          float v = SWIGLU ? silu(acc[ar][t]) * acc[ar + kGemvRows][t] : acc[ar][t];
          const int entry = base + c0 + t;
          const int64_t orow = a.out_by_route ? entry : (a.tok ? a.tok[entry] : entry);
          if (a.bias) v += a.bias[n];
          if (a.resid) v += __bfloat162float(a.resid[orow * a.ldr + n]);
          a.out[orow * a.ldo + n] = __float2bfloat16(v);
        }
      }
  }
}

// ------------------------------------------------------------------------------------------------ attention
constexpr int kKeyChunk = 64;
constexpr int kMaxG = 8;

template <int D>
__global__ void __launch_bounds__(128) decode_attn_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc,
                                                          const bf16* __restrict__ vc, const int* __restrict__ lens,
                                                          int Hq, int Hkv, int Lmax, float scale,
                                                          float* __restrict__ part_o, float* __restrict__ part_ml,
                                                          int chunks, int* __restrict__ tickets,
                                                          bf16* __restrict__ out) {
  constexpr int LPK = D / 8;        // lanes per key (8 head dims each)
  constexpr int KPS = 32 / LPK;     // keys per warp step
  constexpr int STEPS = 16 / KPS;   // a warp owns 16 keys of the chunk
  __shared__ float ps[kMaxG][kKeyChunk];
  __shared__ float po[4][kMaxG][D];
  __shared__ float stats[kMaxG][2];
  __shared__ int s_last;
  griddep_wait();
  griddep_launch();
  const int c = blockIdx.x;
  const int b = blockIdx.y / Hkv, hk = blockIdx.y % Hkv;
  const int G = Hq / Hkv;
  const int len = lens[b];
  const int used = (len + kKeyChunk - 1) / kKeyChunk;
  if (c >= used) return;
  const int k0 = c * kKeyChunk;
  const int nk = min(kKeyChunk, len - k0);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kg = lane / LPK, li = lane % LPK;
  const bf16* kbase = kc + ((static_cast<int64_t>(b) * Hkv + hk) * Lmax + k0) * D + li * 8;
  const bf16* vbase = vc + ((static_cast<int64_t>(b) * Hkv + hk) * Lmax + k0) * D + li * 8;
  uint4 kraw[STEPS];
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int jl = warp * 16 + s * KPS + kg;
    kraw[s] = jl < nk ? __ldg(reinterpret_cast<const uint4*>(kbase + static_cast<int64_t>(jl) * D))
                      : make_uint4(0, 0, 0, 0);
  }
  float qr[kMaxG][8];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g < G) {
      bf16x8_to_float(*reinterpret_cast<const uint4*>(q + (static_cast<int64_t>(b) * Hq + hk * G + g) * D + li * 8),
                      qr[g]);
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[g][e] *= scale;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[g][e] = 0.f;
    }
  }
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int jl = warp * 16 + s * KPS + kg;
    float kv[8];
    bf16x8_to_float(kraw[s], kv);
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g < G) {
        float sc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) sc += qr[g][e] * kv[e];
#pragma unroll
        for (int o = LPK / 2; o > 0; o >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
        if (li == 0 && jl < nk) ps[g][jl] = sc;
      }
    }
  }
  uint4 vraw[STEPS];  // issue the value loads before the softmax
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int jl = warp * 16 + s * KPS + kg;
    vraw[s] = jl < nk ? __ldg(reinterpret_cast<const uint4*>(vbase + static_cast<int64_t>(jl) * D))
                      : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  for (int g = warp; g < G; g += 4) {
    float m = -INFINITY;
    for (int j = lane; j < nk; j += 32) m = fmaxf(m, ps[g][j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < nk; j += 32) {
      const float p = __expf(ps[g][j] - m);
      ps[g][j] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stats[g][0] = m;
      stats[g][1] = l;
    }
  }
  __syncthreads();
  float acc[kMaxG][8];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int jl = warp * 16 + s * KPS + kg;
    if (jl < nk) {
      float vv[8];
      bf16x8_to_float(vraw[s], vv);
#pragma unroll
      for (int g = 0; g < kMaxG; ++g)
        if (g < G) {
          const float p = ps[g][jl];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[g][e] += p * vv[e];
        }
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxG; ++g)
    if (g < G)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = acc[g][e];
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (kg == 0) po[warp][g][li * 8 + e] = v;
      }
  __syncthreads();
  const int64_t pidx = (static_cast<int64_t>(b) * Hq + hk * G) * chunks + c;  // (head hk*G + g, chunk c) at + g*chunks
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    part_o[(pidx + g * chunks) * D + d] = po[0][g][d] + po[1][g][d] + po[2][g][d] + po[3][g][d];
  }
  if (threadIdx.x < G) {
    part_ml[(pidx + threadIdx.x * chunks) * 2] = stats[threadIdx.x][0];
    part_ml[(pidx + threadIdx.x * chunks) * 2 + 1] = stats[threadIdx.x][1];
  }
  // the last chunk block of this (batch, kv head) merges the chunks
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&tickets[blockIdx.y], 1) == used - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    const int64_t hb = (static_cast<int64_t>(b) * Hq + hk * G + g) * chunks;
    float M = -INFINITY;
    for (int cc = 0; cc < used; ++cc) M = fmaxf(M, __ldcg(part_ml + (hb + cc) * 2));
    float L = 0.f, o = 0.f;
    for (int cc = 0; cc < used; ++cc) {
      const float f = __expf(__ldcg(part_ml + (hb + cc) * 2) - M);
      L += f * __ldcg(part_ml + (hb + cc) * 2 + 1);
      o += f * __ldcg(part_o + (hb + cc) * D + d);
    }
    out[(static_cast<int64_t>(b) * Hq + hk * G + g) * D + d] = __float2bfloat16(L > 0.f ? o / L : 0.f);
  }
  if (threadIdx.x == 0) tickets[blockIdx.y] = 0;
}

// Decode attention straight from the QKV GEMV output, with RoPE and the KV-cache append of the new token folded in
// (one launch instead of rope_append + decode_attn_kernel). The cached keys and values of the chunk, which the
// previous kernel does not write, are loaded before the programmatic-launch wait; after it each block rotates its q
// heads (lanes li and li ^ LPK/2 hold the two halves of a rotation pair), and the block whose chunk holds the new
// position rotates the new key, writes key and value into the caches (one writer per batch x kv head) and uses them
// in place of the cache rows. Chunk merge as in decode_attn_kernel.
template <int D>
__global__ void __launch_bounds__(128) decode_attn_rope_kernel(
    const bf16* __restrict__ qkv, const int* __restrict__ pos, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int rope, bf16* __restrict__ kc, bf16* __restrict__ vc, int Hq, int Hkv,
    int Lmax, float scale, float* __restrict__ part_o, float* __restrict__ part_ml, int chunks,
    int* __restrict__ tickets, bf16* __restrict__ out) {
  constexpr int LPK = D / 8;        // lanes per key (8 head dims each)
  constexpr int KPS = 32 / LPK;     // keys per warp step
  constexpr int STEPS = 16 / KPS;   // a warp owns 16 keys of the chunk
  constexpr int HALF = D / 2;
  __shared__ float ps[kMaxG][kKeyChunk];
  __shared__ float po[4][kMaxG][D];
  __shared__ float stats[kMaxG][2];
  __shared__ int s_last;
  const int c = blockIdx.x;
  const int b = blockIdx.y / Hkv, hk = blockIdx.y % Hkv;
  const int G = Hq / Hkv;
  const int p = pos[b];  // written before the step, not by the previous kernel
  const int len = p + 1;
  const int used = (len + kKeyChunk - 1) / kKeyChunk;
  if (c >= used) return;
  const int k0 = c * kKeyChunk;
  const int nk = min(kKeyChunk, len - k0);
  const int jnew = p - k0;  // the new key's slot in this chunk (in range only for the last chunk)
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kg = lane / LPK, li = lane % LPK;
  const int64_t cache_row = (static_cast<int64_t>(b) * Hkv + hk) * Lmax;
  const bf16* kbase = kc + (cache_row + k0) * D + li * 8;
  const bf16* vbase = vc + (cache_row + k0) * D + li * 8;
  // cached keys and values (everything before the new position): independent of the previous kernel
  uint4 kraw[STEPS], vraw[STEPS];
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int jl = warp * 16 + s * KPS + kg;
    const bool cached = jl < nk && jl != jnew;
    kraw[s] = cached ? __ldg(reinterpret_cast<const uint4*>(kbase + static_cast<int64_t>(jl) * D))
                     : make_uint4(0, 0, 0, 0);
    vraw[s] = cached ? __ldg(reinterpret_cast<const uint4*>(vbase + static_cast<int64_t>(jl) * D))
                     : make_uint4(0, 0, 0, 0);
  }
  griddep_wait();
  griddep_launch();
  const int width = (Hq + 2 * Hkv) * D;
  const bf16* row = qkv + static_cast<int64_t>(b) * width;
  // rotation of the 8 dims d = li*8 + e of a head row; the partner dims d +- D/2 live in lane li ^ LPK/2
  auto rotate = [&](float* x) {
    if (!rope) return;
    const bool first = li < LPK / 2;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, x[e], LPK / 2);
      const int j = (li * 8 + e) % HALF;
      const float cs = cos_t[static_cast<int64_t>(p) * HALF + j], sn = sin_t[static_cast<int64_t>(p) * HALF + j];
      x[e] = first ? x[e] * cs - other * sn : x[e] * cs + other * sn;
    }
  };
  float qr[kMaxG][8];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g < G) {
      bf16x8_to_float(*reinterpret_cast<const uint4*>(row + (hk * G + g) * D + li * 8), qr[g]);
      rotate(qr[g]);
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[g][e] *= scale;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[g][e] = 0.f;
    }
  }
  if (jnew >= 0 && jnew < kKeyChunk) {  // block-uniform: this chunk holds the new position
    float kn[8];
    bf16x8_to_float(*reinterpret_cast<const uint4*>(row + (Hq + hk) * D + li * 8), kn);
    rotate(kn);
    uint4 knew;
    knew.x = pack_bf16(kn[0], kn[1]); knew.y = pack_bf16(kn[2], kn[3]);
    knew.z = pack_bf16(kn[4], kn[5]); knew.w = pack_bf16(kn[6], kn[7]);
    const uint4 vnew = *reinterpret_cast<const uint4*>(row + (Hq + Hkv + hk) * D + li * 8);
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      if (warp * 16 + s * KPS + kg == jnew) {  // the LPK lanes of the new key's group
        kraw[s] = knew;
        vraw[s] = vnew;
        *reinterpret_cast<uint4*>(kc + (cache_row + p) * D + li * 8) = knew;
        *reinterpret_cast<uint4*>(vc + (cache_row + p) * D + li * 8) = vnew;
      }
    }
  }
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int jl = warp * 16 + s * KPS + kg;
    float kv[8];
    bf16x8_to_float(kraw[s], kv);
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g < G) {
        float sc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) sc += qr[g][e] * kv[e];
#pragma unroll
        for (int o = LPK / 2; o > 0; o >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
        if (li == 0 && jl < nk) ps[g][jl] = sc;
      }
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += 4) {
    float m = -INFINITY;
    for (int j = lane; j < nk; j += 32) m = fmaxf(m, ps[g][j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < nk; j += 32) {
      const float pv = __expf(ps[g][j] - m);
      ps[g][j] = pv;
      l += pv;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stats[g][0] = m;
      stats[g][1] = l;
    }
  }
  __syncthreads();
  float acc[kMaxG][8];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int jl = warp * 16 + s * KPS + kg;
    if (jl < nk) {
      float vv[8];
      bf16x8_to_float(vraw[s], vv);
#pragma unroll
      for (int g = 0; g < kMaxG; ++g)
        if (g < G) {
          const float pr = ps[g][jl];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[g][e] += pr * vv[e];
        }
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxG; ++g)
    if (g < G)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = acc[g][e];
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (kg == 0) po[warp][g][li * 8 + e] = v;
      }
  __syncthreads();
  const int64_t pidx = (static_cast<int64_t>(b) * Hq + hk * G) * chunks + c;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    part_o[(pidx + g * chunks) * D + d] = po[0][g][d] + po[1][g][d] + po[2][g][d] + po[3][g][d];
  }
  if (threadIdx.x < G) {
    part_ml[(pidx + threadIdx.x * chunks) * 2] = stats[threadIdx.x][0];
    part_ml[(pidx + threadIdx.x * chunks) * 2 + 1] = stats[threadIdx.x][1];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&tickets[blockIdx.y], 1) == used - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    const int64_t hb = (static_cast<int64_t>(b) * Hq + hk * G + g) * chunks;
    float M = -INFINITY;
    for (int cc = 0; cc < used; ++cc) M = fmaxf(M, __ldcg(part_ml + (hb + cc) * 2));
    float L = 0.f, o = 0.f;
    for (int cc = 0; cc < used; ++cc) {
      const float f = __expf(__ldcg(part_ml + (hb + cc) * 2) - M);
      L += f * __ldcg(part_ml + (hb + cc) * 2 + 1);
      o += f * __ldcg(part_o + (hb + cc) * D + d);
    }
    out[(static_cast<int64_t>(b) * Hq + hk * G + g) * D + d] = __float2bfloat16(L > 0.f ? o / L : 0.f);
  }
  if (threadIdx.x == 0) tickets[blockIdx.y] = 0;
}

// qkv [B, (Hq + 2Hkv) * D] for one new token per sequence at position pos[b]: rotate q and k, write q to
// q_out [B, Hq, D] and k, v into the caches [B, Hkv, Lmax, D].
__global__ void __launch_bounds__(256) rope_append_kernel(const bf16* __restrict__ qkv, const int* __restrict__ pos,
                                                          int Hq, int Hkv, int D, int Lmax,
                                                          const float* __restrict__ cos_t,
                                                          const float* __restrict__ sin_t, int rope,
                                                          bf16* __restrict__ q_out, bf16* __restrict__ kc,
                                                          bf16* __restrict__ vc) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x;
  const int p = pos[b];
  const int half = D / 2;
  const int width = (Hq + 2 * Hkv) * D;
  const bf16* row = qkv + static_cast<int64_t>(b) * width;
  for (int i = threadIdx.x; i < (Hq + Hkv) * half; i += blockDim.x) {
    const int h = i / half, j = i % half;
    const float x1 = __bfloat162float(row[h * D + j]);
    const float x2 = __bfloat162float(row[h * D + j + half]);
    float y1 = x1, y2 = x2;
    if (rope) {
      const float c = cos_t[static_cast<int64_t>(p) * half + j];
      const float s = sin_t[static_cast<int64_t>(p) * half + j];
      y1 = x1 * c - x2 * s;
      y2 = x2 * c + x1 * s;
    }
    bf16* o = h < Hq ? q_out + (static_cast<int64_t>(b) * Hq + h) * D
                     : kc + ((static_cast<int64_t>(b) * Hkv + (h - Hq)) * Lmax + p) * D;
    o[j] = __float2bfloat16(y1);
    o[j + half] = __float2bfloat16(y2);
  }
  for (int i = threadIdx.x; i < Hkv * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    vc[((static_cast<int64_t>(b) * Hkv + h) * Lmax + p) * D + d] = row[(Hq + Hkv) * D + h * D + d];
  }
}

// ------------------------------------------------------------------------------------------------ combine + norm
// Block per token t. xin[t] = embedding (tokens given) or the residual stream x[t]; plus, when y is given, the MoE
// output of the previous layer sum_j top_w[t, j] * y[slot[t, j]] (fp32 sum, rounded to bf16 like the residual
// stream). Writes the new residual to x_out (optional) and LayerNorm/RMSNorm(xin) to n_out.
__global__ void __launch_bounds__(256) combine_norm_kernel(const bf16* __restrict__ x, const int64_t* __restrict__ tokens,
                                                           const bf16* __restrict__ tok_emb,
                                                           const bf16* __restrict__ pos_emb,
                                                           const int* __restrict__ positions,
                                                           const bf16* __restrict__ y, const int* __restrict__ slot,
                                                           const float* __restrict__ top_w, int k, int H,
                                                           const float* __restrict__ w, const float* __restrict__ bias,
                                                           float eps, int rms, bf16* __restrict__ x_out,
                                                           bf16* __restrict__ n_out, const float* __restrict__ parts,
                                                           const int* __restrict__ part_step, int part_layer,
                                                           int part_layers, int part_world, int part_tstride) {
  extern __shared__ float v[];  // [H]
  __shared__ float red[2][8];
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bf16* src = tokens ? tok_emb + tokens[t] * H : x + static_cast<int64_t>(t) * H;
  const bf16* prow = (tokens && pos_emb) ? pos_emb + static_cast<int64_t>(positions[t]) * H : nullptr;
  float sum = 0.f;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float val = __bfloat162float(src[h]);
    if (prow) val = __bfloat162float(__float2bfloat16(val + __bfloat162float(prow[h])));
    if (y) {
      float add = 0.f;
      for (int j = 0; j < k; ++j)
        add += top_w[t * k + j] * __bfloat162float(y[static_cast<int64_t>(slot[t * k + j]) * H + h]);
      val = __bfloat162float(__float2bfloat16(val + add));
    } else if (parts) {  // expert-parallel decode: every rank's partial MoE output, summed in rank order
      const int64_t plane = (*part_step & 1) * part_layers + part_layer;
      const float* base = parts + plane * part_world * static_cast<int64_t>(part_tstride) * H;
      float add = 0.f;
      for (int r = 0; r < part_world; ++r) add += base[(static_cast<int64_t>(r) * part_tstride + t) * H + h];
      val = __bfloat162float(__float2bfloat16(val + add));
    }
    if (x_out) x_out[static_cast<int64_t>(t) * H + h] = __float2bfloat16(val);
    v[h] = val;
    sum += val;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[0][warp] = sum;
  __syncthreads();
  float mean = 0.f;
  if (!rms) {
    for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) mean += red[0][i];
    mean /= H;
  }
  float sq = 0.f;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const float d = v[h] - mean;
    sq += d * d;
  }
  sq = warp_sum(sq);
  if (lane == 0) red[1][warp] = sq;
  __syncthreads();
  float var = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) var += red[1][i];
  const float rstd = rsqrtf(var / H + eps);
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float o = (v[h] - mean) * rstd * w[h];
    if (bias) o += bias[h];
    n_out[static_cast<int64_t>(t) * H + h] = __float2bfloat16(o);
  }
}

// ------------------------------------------------------------------------------------------------ routing (decode)
// Grid E blocks: block e writes logits[t, e] = x[t] . wr[e] / temperature for every token (one warp per token). The
// last block to finish (ticket) does, for T <= 64 tokens: softmax, top-k (by probability, or logits + bias),
// renormalised weights; then per-expert lists: cnt[e], off[e] (exclusive prefix), order[off[e] + i] = token of the
// i-th route of expert e (routes in token order), route_slot[t*k + j] = its index in `order`, active = experts with
// routes (ascending, -1 padded to min(E, T*k)). No capacity.
__global__ void __launch_bounds__(256) decode_route_kernel(const bf16* __restrict__ x, const float* __restrict__ wr,
                                                           const float* __restrict__ ebias, int T, int H, int E, int k,
                                                           float temperature, float* __restrict__ glogits,
                                                           int* __restrict__ cnt, int* __restrict__ off,
                                                           int* __restrict__ order, int* __restrict__ route_slot,
                                                           float* __restrict__ top_w, int* __restrict__ active,
                                                           int* __restrict__ ticket, int first, int local) {
  extern __shared__ float sh[];
  __shared__ int s_last;
  const int e_blk = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, warps = blockDim.x / 32;
  const float* wrow = wr + static_cast<int64_t>(e_blk) * H;
  for (int h = threadIdx.x * 32; h < H; h += blockDim.x * 32) prefetch_l2(wrow + h);
  griddep_wait();
  griddep_launch();
  for (int t = warp; t < T; t += warps) {
    float s = 0.f;
    for (int h = lane * 4; h < H; h += 128) {
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(wrow + h));
      const uint2 xr = __ldg(reinterpret_cast<const uint2*>(x + static_cast<int64_t>(t) * H + h));
      const bf16* xb = reinterpret_cast<const bf16*>(&xr);
      s += w4.x * __bfloat162float(xb[0]) + w4.y * __bfloat162float(xb[1]) + w4.z * __bfloat162float(xb[2]) +
           w4.w * __bfloat162float(xb[3]);
    }
    s = warp_sum(s);
    if (lane == 0) glogits[static_cast<int64_t>(t) * E + e_blk] = s / temperature;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1) == E - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* logits = sh;                                    // [T][E]
  int* s_idx = reinterpret_cast<int*>(logits + T * E);   // [T][k]
  int* s_cnt = s_idx + T * k;                            // [E]
  for (int i = threadIdx.x; i < T * E; i += blockDim.x) logits[i] = __ldcg(glogits + i);
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int t = warp; t < T; t += warps) {  // one warp per token: softmax + top-k
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, logits[t * E + e]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int e = lane; e < E; e += 32) sum += __expf(logits[t * E + e] - mx);
    sum = warp_sum(sum);
    float wsum = 0.f;
    float chosen_p[8];
    int chosen_e[8];
    for (int j = 0; j < k; ++j) {
      float best = -INFINITY;
      int be = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        bool used = false;
        for (int i2 = 0; i2 < j; ++i2) used |= (chosen_e[i2] == e);
        if (used) continue;
        const float key = ebias ? logits[t * E + e] + ebias[e] : __expf(logits[t * E + e] - mx) / sum;
        if (key > best || (key == best && e < be)) {
          best = key;
          be = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ob > best || (ob == best && oe < be)) {
          best = ob;
          be = oe;
        }
      }
      chosen_e[j] = be;
      chosen_p[j] = __expf(logits[t * E + be] - mx) / sum;
      wsum += chosen_p[j];
    }
    if (lane == 0)
      for (int j = 0; j < k; ++j) {
        s_idx[t * k + j] = chosen_e[j];
        top_w[t * k + j] = chosen_p[j] / wsum;
      }
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // tiny serial scan: counts, offsets, stable lists, compact list of active experts
    for (int r = 0; r < T * k; ++r) s_cnt[s_idx[r]]++;
    const int slots = min(E, T * k);
    int acc = 0, n_active = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = acc;
      cnt[e] = s_cnt[e];
      acc += s_cnt[e];
      // the active list names the experts this rank holds (all of them unless expert-parallel), relative to `first`
      if (s_cnt[e] > 0 && e >= first && e < first + local && n_active < slots) active[n_active++] = e - first;
      s_cnt[e] = 0;
    }
    for (int i = n_active; i < slots; ++i) active[i] = -1;
    for (int r = 0; r < T * k; ++r) {
      const int e = s_idx[r];
      const int slot = off[e] + s_cnt[e]++;
      order[slot] = r / k;
      route_slot[r] = slot;
    }
    *ticket = 0;
  }
}

template <int FMT, bool SW>
void launch_gemv(const GemvArgs& a, int groups, int grid_groups, cudaStream_t stream) {
  dim3 grid((a.N + kGemvWarps * kGemvRows - 1) / (kGemvWarps * kGemvRows), a.active ? grid_groups : groups);
  if (a.active == nullptr && a.cnt == nullptr)
    launch_pdl(gemv_kernel<FMT, SW, true>, grid, dim3(kGemvWarps * 32), 0, stream, "grouped_gemv", a);
  else
    launch_pdl(gemv_kernel<FMT, SW, false>, grid, dim3(kGemvWarps * 32), 0, stream, "grouped_gemv", a);
}

}  // namespace

// fmt: 0 bf16, 1 int8 (per-row scale), 2 int4 (group-wise scales). swiglu: W holds 2N rows [gate; up].
void grouped_gemv(const bf16* x, int64_t ldx, const void* w, const void* scales, int64_t w_group_bytes,
                  int64_t s_group_elems, int N, int K, int group, int fmt, bool swiglu, const int* tok, const int* off,
                  const int* cnt, int groups, int dense_rows, bf16* out, int64_t ldo, bool out_by_route,
                  const float* bias, const bf16* resid, int64_t ldr, const int* active, int active_slots,
                  cudaStream_t stream) {
  if (K % 32) throw std::runtime_error("grouped_gemv: K must be a multiple of 32");
  if (fmt == 2 && (group % 32 || K % group)) throw std::runtime_error("grouped_gemv: int4 group must divide K, %32");
  if (ldx % 8) throw std::runtime_error("grouped_gemv: x rows must be 16-byte aligned");
  GemvArgs a{x, ldx, static_cast<const uint8_t*>(w), static_cast<const __half*>(scales), w_group_bytes, s_group_elems,
             N, K, group, tok, off, cnt, dense_rows, out, ldo, out_by_route ? 1 : 0, bias, resid, ldr, active};
#define QW_GEMV(F, S) launch_gemv<F, S>(a, groups, active_slots, stream)
  if (fmt == 0) { if (swiglu) QW_GEMV(0, true); else QW_GEMV(0, false); }
  else if (fmt == 1) { if (swiglu) QW_GEMV(1, true); else QW_GEMV(1, false); }
  else if (fmt == 2) { if (swiglu) QW_GEMV(2, true); else QW_GEMV(2, false); }
  else throw std::runtime_error("grouped_gemv: unknown weight format");
#undef QW_GEMV
}

int decode_attn_chunks(int Lmax) { return (Lmax + kKeyChunk - 1) / kKeyChunk; }

void decode_attention(const bf16* q, const bf16* kc, const bf16* vc, const int* lens, int B, int Hq, int Hkv, int D,
                      int Lmax, float scale, float* part_o, float* part_ml, int* tickets, bf16* out,
                      cudaStream_t stream) {
  if (Hq % Hkv || Hq / Hkv > kMaxG) throw std::runtime_error("decode attention: at most 8 q heads per kv head");
  const int chunks = decode_attn_chunks(Lmax);
  dim3 grid(chunks, B * Hkv);
#define QW_ATTN(DIM)                                                                                               \
  launch_pdl(decode_attn_kernel<DIM>, grid, dim3(128), 0, stream, "decode_attention", q, kc, vc, lens, Hq, Hkv, Lmax, \
             scale, part_o, part_ml, chunks, tickets, out)
  if (D == 64) QW_ATTN(64);
  else if (D == 128) QW_ATTN(128);
  else if (D == 32) QW_ATTN(32);
  else throw std::runtime_error("decode attention: head_dim must be 32, 64 or 128");
#undef QW_ATTN
}

void decode_attention_rope(const bf16* qkv, const int* pos, const float* cos_t, const float* sin_t, bool rope,
                           bf16* kc, bf16* vc, int B, int Hq, int Hkv, int D, int Lmax, float scale, float* part_o,
                           float* part_ml, int* tickets, bf16* out, cudaStream_t stream) {
  if (Hq % Hkv || Hq / Hkv > kMaxG) throw std::runtime_error("decode attention: at most 8 q heads per kv head");
  const int chunks = decode_attn_chunks(Lmax);
  dim3 grid(chunks, B * Hkv);
#define QW_ATTN(DIM)                                                                                               \
  launch_pdl(decode_attn_rope_kernel<DIM>, grid, dim3(128), 0, stream, "decode_attention_rope", qkv, pos, cos_t,   \
             sin_t, rope ? 1 : 0, kc, vc, Hq, Hkv, Lmax, scale, part_o, part_ml, chunks, tickets, out)
  if (D == 64) QW_ATTN(64);
  else if (D == 128) QW_ATTN(128);
  else if (D == 32) QW_ATTN(32);
  else throw std::runtime_error("decode attention: head_dim must be 32, 64 or 128");
#undef QW_ATTN
}

void rope_append(const bf16* qkv, const int* pos, int B, int Hq, int Hkv, int D, int Lmax, const float* cos_t,
                 const float* sin_t, bool rope, bf16* q_out, bf16* kc, bf16* vc, cudaStream_t stream) {
  launch_pdl(rope_append_kernel, dim3(B), dim3(256), 0, stream, "rope_append", qkv, pos, Hq, Hkv, D, Lmax, cos_t,
             sin_t, rope ? 1 : 0, q_out, kc, vc);
}

void decode_combine_norm(const bf16* x, const int64_t* tokens, const bf16* tok_emb, const bf16* pos_emb,
                         const int* positions, const bf16* y, const int* slot, const float* top_w, int k, int T, int H,
                         const float* w, const float* bias, float eps, bool rms, bf16* x_out, bf16* n_out,
                         cudaStream_t stream, const float* parts, const int* part_step, int part_layer,
                         int part_layers, int part_world, int part_tstride) {
  if (T == 0) return;
  const size_t smem = static_cast<size_t>(H) * sizeof(float);
  if (smem > 48 * 1024)
    check_cuda(cudaFuncSetAttribute(combine_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)), "combine_norm smem");
  launch_pdl(combine_norm_kernel, dim3(T), dim3(256), smem, stream, "decode_combine_norm", x, tokens, tok_emb,
             pos_emb, positions, y, slot, top_w, k, H, w, bias, eps, rms ? 1 : 0, x_out, n_out, parts, part_step,
             part_layer, part_layers, part_world, part_tstride);
}

void decode_route(const bf16* x, const float* wr, const float* ebias, int T, int H, int E, int k, float temperature,
                  float* logits, int* cnt, int* off, int* order, int* route_slot, float* top_w, int* active,
                  int* ticket, cudaStream_t stream, int first, int local) {
  if (T > 64 || k > 8) throw std::runtime_error("decode_route: at most 64 tokens and top-8");
  if (H % 128) throw std::runtime_error("decode_route: hidden size must be a multiple of 128");
  const size_t smem = static_cast<size_t>(T) * E * sizeof(float) + (static_cast<size_t>(T) * k + E) * sizeof(int);
  check_cuda(cudaFuncSetAttribute(decode_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(std::max<size_t>(smem, 1024))), "decode_route smem");
  launch_pdl(decode_route_kernel, dim3(E), dim3(256), smem, stream, "decode_route", x, wr, ebias, T, H, E, k,
             temperature, logits, cnt, off, order, route_slot, top_w, active, ticket, first, local < 0 ? E : local);
}

int decode_status(bool clear) { return read_status_word(clear); }



// ------------------------------------------------------------------------------------------------ dequantisation
// bf16 copy of packed weight rows, for the tensor-core GEMMs that serve many tokens at once (prefill): int4 (fmt 2,
// two values per byte, low nibble = even column, value = (nibble - 8) * scale of its group of `group` columns) or
// int8 (fmt 1, one scale per row). One thread writes 8 consecutive bf16 (one 16-byte store).
namespace {
__global__ void __launch_bounds__(256) dequant_rows_kernel(const uint8_t* __restrict__ q, const __half* __restrict__ s,
                                                           int64_t rows, int K, int group, int fmt,
                                                           bf16* __restrict__ out) {
  const int vecs_per_row = K / 8;
  const int64_t total = rows * vecs_per_row;
  const int spr = fmt == 2 ? K / group : 1;  // scales per row
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vecs_per_row;
    const int k0 = static_cast<int>(i % vecs_per_row) * 8;
    const float scale = __half2float(s[r * spr + (fmt == 2 ? k0 / group : 0)]);
    float v[8];
    if (fmt == 2) {
      const uint32_t packed = *reinterpret_cast<const uint32_t*>(q + r * (K / 2) + k0 / 2);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = static_cast<float>(static_cast<int>((packed >> (4 * j)) & 0xFu) - 8) * scale;
    } else {
      const uint2 packed = *reinterpret_cast<const uint2*>(q + r * K + k0);
      const int8_t* b = reinterpret_cast<const int8_t*>(&packed);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = static_cast<float>(b[j]) * scale;
    }
    uint4 w;
    w.x = pack_bf16(v[0], v[1]);
    w.y = pack_bf16(v[2], v[3]);
    w.z = pack_bf16(v[4], v[5]);
    w.w = pack_bf16(v[6], v[7]);
    *reinterpret_cast<uint4*>(out + r * K + k0) = w;
  }
}
}  // namespace

void dequant_rows(const void* q, const void* scales, int64_t rows, int K, int group, int fmt, bf16* out,
                  cudaStream_t stream) {
  if (rows == 0) return;
  if (K % 8 || (fmt == 2 && (group % 8 || K % group))) throw std::runtime_error("dequant_rows: K / group layout");
  const int64_t total = rows * (K / 8);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(148 * 16, (total + 255) / 256)));
  dequant_rows_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(q), static_cast<const __half*>(scales),
                                                rows, K, group, fmt, out);
  check_cuda(cudaGetLastError(), "dequant_rows");
}

}  // namespace qw
