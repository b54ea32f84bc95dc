// Causal flash attention (forward + deterministic backward) with grouped-query attention, head_dim 32, 64 or 128.
//
// Tensors are token-major, exactly as the QKV GEMM writes them: q/k/v/o rows are tokens (b*S + s), a head's D
// values sit at column h*D of a row with leading dimension ld (so packed [T, (Hq+2Hkv)*D] QKV is read in place).
// lse is [B, Hq, S] fp32 (natural log).
//
// Forward: one CTA = 128 queries (8 warps x 16 rows) of one (batch, q-head), key tiles of 64 double-buffered with
// cp.async into 128-byte-XOR-swizzled shared memory; S = QK^T and O += PV on bf16 tensor cores (mma.sync
// m16n8k16, fp32 accumulate) with the online softmax in registers (exp2 domain).
// Backward (no atomics, bit-reproducible): kernel 1 owns a key tile and loops over query tiles and the q-heads of
// its kv group to accumulate dK, dV; kernel 2 owns a query tile and loops over key tiles to accumulate dQ.
#include <algorithm>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "launchers.h"

namespace qw {
namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// element offset of (row, 8-element chunk) in a [rows][D] tile with the chunk index XOR-swizzled by row % 8
template <int D>
__device__ __forceinline__ int swz(int row, int chunk) {
  constexpr int kMask = (D / 8 < 8 ? D / 8 : 8) - 1;
  return row * D + ((chunk ^ (row & kMask)) << 3);
}

// async copy of `rows` x D tile from token-major global memory (rows past `valid_rows` are zero-filled)
template <int D, int ROWS, int THREADS>
__device__ __forceinline__ void load_tile(bf16* tile, const bf16* g, int64_t ld, int valid_rows) {
  constexpr int CHUNKS = D / 8;
  for (int i = threadIdx.x; i < ROWS * CHUNKS; i += THREADS) {
    const int r = i / CHUNKS, c = i % CHUNKS;
    const bool ok = r < valid_rows;
    cp_async16(tile + swz<D>(r, c), g + (ok ? static_cast<int64_t>(r) * ld + c * 8 : 0), ok);
  }
}

// A fragments (16 rows x D) of a [rows][D] smem tile starting at row r0
template <int D>
__device__ __forceinline__ void load_a_frags(const bf16* tile, int r0, uint32_t (*frag)[4]) {
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int row = r0 + (lane % 8) + ((lane / 8) % 2) * 8;
    const int chunk = 2 * ks + lane / 16;
    ldsm_x4(smem_u32(tile + swz<D>(row, chunk)), frag[ks][0], frag[ks][1], frag[ks][2], frag[ks][3]);
  }
}

// acc[16 x 8*NT] += A(16 x D, registers) * B^T where B rows = tile rows n0.. (B[k=d][n=row] = tile[row][d])
template <int D, int NT>
__device__ __forceinline__ void mma_a_regs_b_rows(float (*acc)[4], const uint32_t (*a)[4], const bf16* tile, int n0) {
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      const int row = n0 + nt * 8 + (lane % 8) + (lane / 16) * 8;
      const int chunk = 2 * ks + (lane / 8) % 2;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(tile + swz<D>(row, chunk)), b0, b1, b2, b3);
      mma16816(acc[nt], a[ks], b0, b1);
      mma16816(acc[nt + 1], a[ks], b2, b3);
    }
  }
}

// acc[16 x D] += P(16 x 16*KS, from C-layout registers) * tile[k0 + key][d]   (tile read transposed)
template <int D, int KS>
__device__ __forceinline__ void mma_p_tile(float (*acc)[4], const float (*p)[4], const bf16* tile, int k0) {
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    uint32_t a[4];
    a[0] = pack_bf16(p[2 * kk][0], p[2 * kk][1]);
    a[1] = pack_bf16(p[2 * kk][2], p[2 * kk][3]);
    a[2] = pack_bf16(p[2 * kk + 1][0], p[2 * kk + 1][1]);
    a[3] = pack_bf16(p[2 * kk + 1][2], p[2 * kk + 1][3]);
#pragma unroll
    for (int dt = 0; dt < D / 8; dt += 2) {
      const int row = k0 + kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
      const int chunk = dt + lane / 16;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(smem_u32(tile + swz<D>(row, chunk)), b0, b1, b2, b3);
      mma16816(acc[dt], a, b0, b1);
      mma16816(acc[dt + 1], a, b2, b3);
    }
  }
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ------------------------------------------------------------------------------------------------ forward
template <int D>
__global__ void __launch_bounds__(256) flash_fwd_kernel(const bf16* __restrict__ q, int64_t ldq,
                                                        const bf16* __restrict__ k, int64_t ldk,
                                                        const bf16* __restrict__ v, int64_t ldv, bf16* __restrict__ o,
                                                        int64_t ldo, float* __restrict__ lse, int S, int Hq, int Hkv,
                                                        float scale) {
  constexpr int BR = 128, BC = 64, NT = BC / 8, DT = D / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  bf16* sq = reinterpret_cast<bf16*>(smem_raw);
  bf16* sk = sq + BR * D;
  bf16* sv = sk + 2 * BC * D;
  const int qb = gridDim.x - 1 - blockIdx.x;  // heaviest (most keys) tiles first
  const int bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hkv);
  const int q0 = qb * BR;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t tok0 = static_cast<int64_t>(b) * S;
  const bf16* qg = q + (tok0 + q0) * ldq + h * D;
  const bf16* kg = k + tok0 * ldk + hk * D;
  const bf16* vg = v + tok0 * ldv + hk * D;

  load_tile<D, BR, 256>(sq, qg, ldq, S - q0);
  const int kv_end = min(S, q0 + BR);
  const int nkb = (kv_end + BC - 1) / BC;
  load_tile<D, BC, 256>(sk, kg, ldk, S);
  load_tile<D, BC, 256>(sv, vg, ldv, S);
  cp_commit();

  uint32_t qf[D / 16][4];
  float acc_o[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) acc_o[i][0] = acc_o[i][1] = acc_o[i][2] = acc_o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const float sl2 = scale * kLog2e;
  const int row_a = q0 + warp * 16 + lane / 4;  // query index of accumulator rows (and +8)

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_tile<D, BC, 256>(sk + (buf ^ 1) * BC * D, kg + static_cast<int64_t>(kb + 1) * BC * ldk, ldk,
                            S - (kb + 1) * BC);
      load_tile<D, BC, 256>(sv + (buf ^ 1) * BC * D, vg + static_cast<int64_t>(kb + 1) * BC * ldv, ldv,
                            S - (kb + 1) * BC);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) load_a_frags<D>(sq, warp * 16, qf);
    const bf16* tk = sk + buf * BC * D;
    const bf16* tv = sv + buf * BC * D;
    float s[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    mma_a_regs_b_rows<D, NT>(s, qf, tk, 0);
    // scale, mask, running max
    const int key0 = kb * BC;
    const bool diag = key0 + BC > q0 + warp * 16;
    float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = key0 + nt * 8 + (lane % 4) * 2 + (j & 1);
        const int qi = row_a + (j >> 1) * 8;
        float x = s[nt][j] * sl2;
        if ((diag && key > qi) || key >= S) x = -INFINITY;
        s[nt][j] = x;
        mx[j >> 1] = fmaxf(mx[j >> 1], x);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], base[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      base[r] = (mx[r] == -INFINITY) ? 0.f : mx[r];
      alpha[r] = exp2f(m_run[r] - base[r]);
      m_run[r] = mx[r];
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = exp2f(s[nt][j] - base[j >> 1]);
        s[nt][j] = pv;
        rs[j >> 1] += pv;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * alpha[r] + rs[r];
#pragma unroll
    for (int dt = 0; dt < DT; ++dt) {
      acc_o[dt][0] *= alpha[0]; acc_o[dt][1] *= alpha[0];
      acc_o[dt][2] *= alpha[1]; acc_o[dt][3] *= alpha[1];
    }
    mma_p_tile<D, BC / 16>(acc_o, s, tv, 0);
    __syncthreads();
  }
  // finalise: quad-reduce row sums, normalise, lse
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  float inv[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) inv[r] = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
  // stage O through the (now free) Q tile for coalesced stores
  bf16* so = sq;
#pragma unroll
  for (int dt = 0; dt < DT; ++dt) {
    const int col = dt * 8 + (lane % 4) * 2;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = warp * 16 + lane / 4 + r * 8;
      const uint32_t packed = pack_bf16(acc_o[dt][2 * r] * inv[r], acc_o[dt][2 * r + 1] * inv[r]);
      *reinterpret_cast<uint32_t*>(so + swz<D>(row, col / 8) + (col % 8)) = packed;
    }
  }
  if (lane % 4 == 0) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int qi = row_a + r * 8;
      if (qi < S) lse[(static_cast<int64_t>(b) * Hq + h) * S + qi] = (m_run[r] + log2f(l_run[r])) * kLn2;
    }
  }
  __syncthreads();
  constexpr int CH = D / 8;
  for (int i = threadIdx.x; i < BR * CH; i += 256) {
    const int r = i / CH, c = i % CH;
    if (q0 + r < S)
      *reinterpret_cast<uint4*>(o + (tok0 + q0 + r) * ldo + h * D + c * 8) =
          *reinterpret_cast<const uint4*>(so + swz<D>(r, c));
  }
}

// ------------------------------------------------------------------------------------------------ backward prep
// delta[b,h,s] = sum_d dO * O
__global__ void attn_delta_kernel(const bf16* __restrict__ o, int64_t ldo, const bf16* __restrict__ dout,
                                  int64_t lddo, float* __restrict__ delta, int B, int S, int Hq, int D) {
  const int warps = blockDim.x / 32;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (idx >= static_cast<int64_t>(B) * S * Hq) return;
  const int64_t tok = idx / Hq;
  const int h = static_cast<int>(idx % Hq);
  float s = 0.f;
  for (int d = lane; d < D; d += 32)
    s += __bfloat162float(o[tok * ldo + h * D + d]) * __bfloat162float(dout[tok * lddo + h * D + d]);
  s = warp_sum(s);
  if (lane == 0) {
    const int b = static_cast<int>(tok / S), sidx = static_cast<int>(tok % S);
    delta[(static_cast<int64_t>(b) * Hq + h) * S + sidx] = s;
  }
}

// delta = rowsum(dO * O) with 16-byte loads: CPR = D / 8 consecutive lanes share a (token, head) row, one 8-wide
// chunk each (16-byte aligned rows, D in {32, 64, 128})
template <int CPR>
__global__ void __launch_bounds__(256) attn_delta_vec_kernel(const bf16* __restrict__ o, int64_t ldo,
                                                             const bf16* __restrict__ dout, int64_t lddo,
                                                             float* __restrict__ delta, int B, int S, int Hq) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t idx = t / CPR;  // (token, head) row
  const int c = static_cast<int>(t % CPR);
  const bool live = idx < static_cast<int64_t>(B) * S * Hq;
  float s = 0.f;
  if (live) {
    const int64_t tok = idx / Hq;
    const int h = static_cast<int>(idx % Hq);
    const uint4 a = *reinterpret_cast<const uint4*>(o + tok * ldo + (h * CPR + c) * 8);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + tok * lddo + (h * CPR + c) * 8);
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __bfloat1622float2(a2[i]), y = __bfloat1622float2(g2[i]);
      s = fmaf(x.x, y.x, fmaf(x.y, y.y, s));
    }
  }
#pragma unroll
  for (int off = CPR / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (live && c == 0) {
    const int64_t tok = idx / Hq;
    const int h = static_cast<int>(idx % Hq);
    const int b = static_cast<int>(tok / S), sidx = static_cast<int>(tok % S);
    delta[(static_cast<int64_t>(b) * Hq + h) * S + sidx] = s;
  }
}

// ------------------------------------------------------------------------------------------------ dK, dV
// CTA = 64 keys (4 warps x 16) of one (batch, kv-head); loops over the group's q-heads and the query tiles.
template <int D, int BR>
__global__ void __launch_bounds__(128) flash_bwd_dkdv_kernel(
    const bf16* __restrict__ q, int64_t ldq, const bf16* __restrict__ k, int64_t ldk, const bf16* __restrict__ v,
    int64_t ldv, const bf16* __restrict__ dout, int64_t lddo, const float* __restrict__ lse,
    const float* __restrict__ delta, bf16* __restrict__ dk, int64_t lddk, bf16* __restrict__ dv, int64_t lddv, int S,
    int Hq, int Hkv, float scale) {
  constexpr int BC = 64, NT = BR / 8, DT = D / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  bf16* sk = reinterpret_cast<bf16*>(smem_raw);
  bf16* sv = sk + BC * D;
  bf16* sq = sv + BC * D;          // [2][BR][D]
  bf16* sdo = sq + 2 * BR * D;     // [2][BR][D]
  float* slse = reinterpret_cast<float*>(sdo + 2 * BR * D);  // [2][BR]
  float* sdelta = slse + 2 * BR;                              // [2][BR]
  const int kb = gridDim.x - 1 - blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / Hkv, hk = bh % Hkv;
  const int group = Hq / Hkv;
  const int k0 = kb * BC;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t tok0 = static_cast<int64_t>(b) * S;
  load_tile<D, BC, 128>(sk, k + (tok0 + k0) * ldk + hk * D, ldk, S - k0);
  load_tile<D, BC, 128>(sv, v + (tok0 + k0) * ldv + hk * D, ldv, S - k0);
  cp_commit();
  float acc_dk[DT][4], acc_dv[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc_dk[i][j] = acc_dv[i][j] = 0.f;
  const float sl2 = scale * kLog2e;
  const int first_qb = k0 / BR;
  const int nqb = (S + BR - 1) / BR;
  const int iters_per_head = nqb - first_qb;
  const int total = iters_per_head * group;
  auto issue = [&](int it, int buf) {
    const int hh = hk * group + it / iters_per_head;
    const int qb = first_qb + it % iters_per_head;
    const int qs = qb * BR;
    load_tile<D, BR, 128>(sq + buf * BR * D, q + (tok0 + qs) * ldq + hh * D, ldq, S - qs);
    load_tile<D, BR, 128>(sdo + buf * BR * D, dout + (tok0 + qs) * lddo + hh * D, lddo, S - qs);
    for (int i = threadIdx.x; i < BR; i += 128) {
      const int qi = qs + i;
      const int64_t li = (static_cast<int64_t>(b) * Hq + hh) * S + qi;
      slse[buf * BR + i] = qi < S ? lse[li] * kLog2e : 0.f;
      sdelta[buf * BR + i] = qi < S ? delta[li] : 0.f;
    }
  };
  issue(0, 0);
  cp_commit();
  uint32_t kf[D / 16][4], vf[D / 16][4];
  const int key_a = k0 + warp * 16 + lane / 4;  // key index of accumulator rows (and +8)
  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    if (it + 1 < total) {
      issue(it + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (it == 0) {
      load_a_frags<D>(sk, warp * 16, kf);
      load_a_frags<D>(sv, warp * 16, vf);
    }
    const int qs = (first_qb + it % iters_per_head) * BR;
    const bf16* tq = sq + buf * BR * D;
    const bf16* tdo = sdo + buf * BR * D;
    const float* tl = slse + buf * BR;
    const float* td = sdelta + buf * BR;
    // S^T = K Q^T  (rows = keys, cols = queries)
    float st[NT][4], dpt[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) st[i][j] = dpt[i][j] = 0.f;
    mma_a_regs_b_rows<D, NT>(st, kf, tq, 0);
    mma_a_regs_b_rows<D, NT>(dpt, vf, tdo, 0);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int qcol = nt * 8 + (lane % 4) * 2 + (j & 1);
        const int qi = qs + qcol;
        const int key = key_a + (j >> 1) * 8;
        float p = exp2f(st[nt][j] * sl2 - tl[qcol]);
        if (qi < key || qi >= S || key >= S) p = 0.f;
        st[nt][j] = p;                                // P^T
        dpt[nt][j] = p * (dpt[nt][j] - td[qcol]);      // dS^T
      }
    mma_p_tile<D, BR / 16>(acc_dv, st, tdo, 0);
    mma_p_tile<D, BR / 16>(acc_dk, dpt, tq, 0);
    __syncthreads();
  }
  // write dK (scaled) and dV
#pragma unroll
  for (int dt = 0; dt < DT; ++dt) {
    const int col = dt * 8 + (lane % 4) * 2;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int key = key_a + r * 8;
      if (key >= S) continue;
      *reinterpret_cast<uint32_t*>(dk + (tok0 + key) * lddk + hk * D + col) =
          pack_bf16(acc_dk[dt][2 * r] * scale, acc_dk[dt][2 * r + 1] * scale);
      *reinterpret_cast<uint32_t*>(dv + (tok0 + key) * lddv + hk * D + col) =
          pack_bf16(acc_dv[dt][2 * r], acc_dv[dt][2 * r + 1]);
    }
  }
}

// ------------------------------------------------------------------------------------------------ dQ
// CTA = 64 queries (4 warps x 16) of one (batch, q-head); loops over key tiles up to the diagonal.
template <int D, int BC>
__global__ void __launch_bounds__(128) flash_bwd_dq_kernel(
    const bf16* __restrict__ q, int64_t ldq, const bf16* __restrict__ k, int64_t ldk, const bf16* __restrict__ v,
    int64_t ldv, const bf16* __restrict__ dout, int64_t lddo, const float* __restrict__ lse,
    const float* __restrict__ delta, bf16* __restrict__ dq, int64_t lddq, int S, int Hq, int Hkv, float scale) {
  constexpr int BR = 64, NT = BC / 8, DT = D / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  bf16* sq = reinterpret_cast<bf16*>(smem_raw);
  bf16* sdo = sq + BR * D;
  bf16* sk = sdo + BR * D;   // [2][BC][D]
  bf16* sv = sk + 2 * BC * D;  // [2][BC][D]
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq;
  const int hk = h / (Hq / Hkv);
  const int q0 = qb * BR;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t tok0 = static_cast<int64_t>(b) * S;
  load_tile<D, BR, 128>(sq, q + (tok0 + q0) * ldq + h * D, ldq, S - q0);
  load_tile<D, BR, 128>(sdo, dout + (tok0 + q0) * lddo + h * D, lddo, S - q0);
  const int kv_end = min(S, q0 + BR);
  const int nkb = (kv_end + BC - 1) / BC;
  load_tile<D, BC, 128>(sk, k + tok0 * ldk + hk * D, ldk, S);
  load_tile<D, BC, 128>(sv, v + tok0 * ldv + hk * D, ldv, S);
  cp_commit();
  const int row_a = q0 + warp * 16 + lane / 4;
  float lse2[2], dl[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = row_a + r * 8;
    const int64_t li = (static_cast<int64_t>(b) * Hq + h) * S + qi;
    lse2[r] = qi < S ? lse[li] * kLog2e : 0.f;
    dl[r] = qi < S ? delta[li] : 0.f;
  }
  uint32_t qf[D / 16][4], df[D / 16][4];
  float acc[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const float sl2 = scale * kLog2e;
  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_tile<D, BC, 128>(sk + (buf ^ 1) * BC * D, k + (tok0 + (kb + 1) * BC) * ldk + hk * D, ldk, S - (kb + 1) * BC);
      load_tile<D, BC, 128>(sv + (buf ^ 1) * BC * D, v + (tok0 + (kb + 1) * BC) * ldv + hk * D, ldv, S - (kb + 1) * BC);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
      load_a_frags<D>(sq, warp * 16, qf);
      load_a_frags<D>(sdo, warp * 16, df);
    }
    const bf16* tk = sk + buf * BC * D;
    const bf16* tv = sv + buf * BC * D;
    float s[NT][4], dp[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.f;
    mma_a_regs_b_rows<D, NT>(s, qf, tk, 0);
    mma_a_regs_b_rows<D, NT>(dp, df, tv, 0);
    const int key0 = kb * BC;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = key0 + nt * 8 + (lane % 4) * 2 + (j & 1);
        const int qi = row_a + (j >> 1) * 8;
        float p = exp2f(s[nt][j] * sl2 - lse2[j >> 1]);
        if (key > qi || key >= S || qi >= S) p = 0.f;
        s[nt][j] = p * (dp[nt][j] - dl[j >> 1]);  // dS
      }
    mma_p_tile<D, BC / 16>(acc, s, tk, 0);
    __syncthreads();
  }
#pragma unroll
  for (int dt = 0; dt < DT; ++dt) {
    const int col = dt * 8 + (lane % 4) * 2;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int qi = row_a + r * 8;
      if (qi >= S) continue;
      *reinterpret_cast<uint32_t*>(dq + (tok0 + qi) * lddq + h * D + col) =
          pack_bf16(acc[dt][2 * r] * scale, acc[dt][2 * r + 1] * scale);
    }
  }
}

template <typename K>
void set_smem(K kernel, size_t bytes) {
  check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
             "attention smem");
}

}  // namespace

void flash_attn_fwd(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, bf16* o,
                    int64_t ldo, float* lse, int B, int S, int Hq, int Hkv, int D, float scale, cudaStream_t stream) {
  if (B == 0 || S == 0) return;
  // head_dim 64 and 128 run on the tcgen05 kernel (attention_fwd_tc.cu); QW_ATTN_FWD=mma keeps the mma.sync kernels
  // below (and head_dim 32 always uses them)
  static const bool use_mma = [] {
    const char* e = std::getenv("QW_ATTN_FWD");
    return e && std::string(e) == "mma";
  }();
  if ((D == 64 || D == 128) && !use_mma) {
    flash_attn_fwd_tc(q, ldq, k, ldk, v, ldv, o, ldo, lse, B, S, Hq, Hkv, D, scale, stream);
    return;
  }
  dim3 grid((S + 127) / 128, B * Hq);
  if (D == 32) {
    const size_t smem = (128 + 4 * 64) * 32 * sizeof(bf16);
    set_smem(flash_fwd_kernel<32>, smem);
    flash_fwd_kernel<32><<<grid, 256, smem, stream>>>(q, ldq, k, ldk, v, ldv, o, ldo, lse, S, Hq, Hkv, scale);
  } else if (D == 64) {
    const size_t smem = (128 + 4 * 64) * 64 * sizeof(bf16);
    set_smem(flash_fwd_kernel<64>, smem);
    flash_fwd_kernel<64><<<grid, 256, smem, stream>>>(q, ldq, k, ldk, v, ldv, o, ldo, lse, S, Hq, Hkv, scale);
  } else if (D == 128) {
    const size_t smem = (128 + 4 * 64) * 128 * sizeof(bf16);
    set_smem(flash_fwd_kernel<128>, smem);
    flash_fwd_kernel<128><<<grid, 256, smem, stream>>>(q, ldq, k, ldk, v, ldv, o, ldo, lse, S, Hq, Hkv, scale);
  } else {
    throw std::runtime_error("flash attention: head_dim must be 32, 64 or 128");
  }
  check_cuda(cudaGetLastError(), "flash_attn_fwd");
}

void flash_attn_bwd(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, const bf16* o,
                    int64_t ldo, const bf16* dout, int64_t lddo, const float* lse, float* delta, bf16* dq,
                    int64_t lddq, bf16* dk, int64_t lddk, bf16* dv, int64_t lddv, int B, int S, int Hq, int Hkv, int D,
                    float scale, cudaStream_t stream) {
  if (B == 0 || S == 0) return;
  const int64_t rows = static_cast<int64_t>(B) * S * Hq;
  const bool vec = (D == 32 || D == 64 || D == 128) && (ldo * 2) % 16 == 0 && (lddo * 2) % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(o) & 15) == 0 && (reinterpret_cast<uintptr_t>(dout) & 15) == 0;
  if (vec) {
    const int64_t threads = rows * (D / 8);
    const int blocks = static_cast<int>((threads + 255) / 256);
    if (D == 64) attn_delta_vec_kernel<8><<<blocks, 256, 0, stream>>>(o, ldo, dout, lddo, delta, B, S, Hq);
    else if (D == 128) attn_delta_vec_kernel<16><<<blocks, 256, 0, stream>>>(o, ldo, dout, lddo, delta, B, S, Hq);
    else attn_delta_vec_kernel<4><<<blocks, 256, 0, stream>>>(o, ldo, dout, lddo, delta, B, S, Hq);
  } else {
    attn_delta_kernel<<<static_cast<int>((rows + 7) / 8), 256, 0, stream>>>(o, ldo, dout, lddo, delta, B, S, Hq, D);
  }
  // head_dim 64 / 128 run on the tcgen05 kernels (attention_tc.cu); QW_ATTN_BWD=mma keeps the mma.sync kernels
  // below for comparison
  static const bool use_mma = [] {
    const char* e = std::getenv("QW_ATTN_BWD");
    return e && std::string(e) == "mma";
  }();
  if ((D == 64 || D == 128) && !use_mma) {
    check_cuda(cudaGetLastError(), "attn_delta");
    flash_attn_bwd_tc(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dq, lddq, dk, lddk, dv, lddv, B, S, Hq, Hkv, D,
                      scale, stream);
    return;
  }
  dim3 grid_kv((S + 63) / 64, B * Hkv);
  dim3 grid_q((S + 63) / 64, B * Hq);
  if (D == 32) {
    constexpr int BR = 64, BC = 64;
    const size_t smem_kv = (2 * 64 + 4 * BR) * 32 * sizeof(bf16) + 4 * BR * sizeof(float);
    set_smem(flash_bwd_dkdv_kernel<32, BR>, smem_kv);
    flash_bwd_dkdv_kernel<32, BR><<<grid_kv, 128, smem_kv, stream>>>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dk,
                                                                     lddk, dv, lddv, S, Hq, Hkv, scale);
    const size_t smem_q = (2 * 64 + 4 * BC) * 32 * sizeof(bf16);
    set_smem(flash_bwd_dq_kernel<32, BC>, smem_q);
    flash_bwd_dq_kernel<32, BC><<<grid_q, 128, smem_q, stream>>>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dq,
                                                                  lddq, S, Hq, Hkv, scale);
  } else if (D == 64) {
    constexpr int BR = 64, BC = 64;
    const size_t smem_kv = (2 * 64 + 4 * BR) * 64 * sizeof(bf16) + 4 * BR * sizeof(float);
    set_smem(flash_bwd_dkdv_kernel<64, BR>, smem_kv);
    flash_bwd_dkdv_kernel<64, BR><<<grid_kv, 128, smem_kv, stream>>>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dk,
                                                                     lddk, dv, lddv, S, Hq, Hkv, scale);
    const size_t smem_q = (2 * 64 + 4 * BC) * 64 * sizeof(bf16);
    set_smem(flash_bwd_dq_kernel<64, BC>, smem_q);
    flash_bwd_dq_kernel<64, BC><<<grid_q, 128, smem_q, stream>>>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dq,
                                                                  lddq, S, Hq, Hkv, scale);
  } else if (D == 128) {
    constexpr int BR = 32, BC = 32;
    const size_t smem_kv = (2 * 64 + 4 * BR) * 128 * sizeof(bf16) + 4 * BR * sizeof(float);
    set_smem(flash_bwd_dkdv_kernel<128, BR>, smem_kv);
    flash_bwd_dkdv_kernel<128, BR><<<grid_kv, 128, smem_kv, stream>>>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta,
                                                                      dk, lddk, dv, lddv, S, Hq, Hkv, scale);
    const size_t smem_q = (2 * 64 + 4 * BC) * 128 * sizeof(bf16);
    set_smem(flash_bwd_dq_kernel<128, BC>, smem_q);
    flash_bwd_dq_kernel<128, BC><<<grid_q, 128, smem_q, stream>>>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dq,
                                                                   lddq, S, Hq, Hkv, scale);
  } else {
    throw std::runtime_error("flash attention: head_dim must be 32, 64 or 128");
  }
  check_cuda(cudaGetLastError(), "flash_attn_bwd");
}

int attention_status(bool clear) { return read_status_word(clear); }

}  // namespace qw
