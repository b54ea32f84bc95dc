// Causal flash-attention forward on the Blackwell tensor cores (head_dim 64 and 128): tcgen05.mma with TMEM
// accumulators, Q/K/V staged by TMA into 128-byte-swizzled shared memory, grouped-query attention read in place from
// the packed QKV rows.
//
// One CTA owns 256 queries of one (batch, q-head) as two 128-row Q tiles, and walks the KT-key K/V tiles up to the
// diagonal (KT = 128 keys at head_dim 64; 64 keys at head_dim 128, so that S, O and P of both tiles fit the 512
// TMEM columns). Each Q tile has its own softmax warpgroup, so while one group turns its scores into probabilities
// the tensor core works on the other group's tiles (ping-pong):
//
//   S_g  = Q_g K_j^T                       (TMEM, 128 x KT fp32 per group; Q and K from shared memory)
//   P_g  = exp2(S_g * scale*log2e - m_g)   (softmax warps, packed f16x2 exponentials -> bf16, stored to TMEM)
//   O_g += P_g V_j                          (TMEM, 128 x D fp32 per group; A = P_g read from TMEM, B = V_j from
//                                           shared memory)
//
// Shared-memory bandwidth (128 B per clock) is what an M = 128, N <= 128 MMA with both operands in shared memory
// runs into: P in shared memory cost a store and a re-read of 32 KB per group and tile on top of the operand reads.
// With P in TMEM the P V MMA reads only V from shared memory.
//
// Lazy rescaling: m_g is the row maximum the accumulator O_g is expressed against. A new tile only moves it when its
// own maximum exceeds m_g by more than 2^8 (so probabilities stay below 256, well inside bf16 and fp32 range);
// then the warp reads O_g out of TMEM, scales it by 2^(m_old - m_new) and writes it back before the next P V
// accumulates. After the first few tiles of a row this almost never happens, so the softmax touches each score once
// (one TMEM read of the row) and never waits for the previous P V except to reuse the P buffer. At the end
// O_g / l is stored in bf16 and lse = ln(sum exp(scale * s)) in fp32 (the backward's input).
//
// Roles (320 threads, one CTA per SM — the shared-memory request guarantees it, so the 512 TMEM columns never
// contend):
//   warp 0      TMA: both Q tiles once, then K_j | V_j through a ring of stages.
//   warp 1      MMA issuer (one thread), polling: per group, S_g(j+1) as soon as tile j+1 has landed and the group
//               has read S_g(j) out of TMEM (so the next scores are computed while the group exponentiates), and
//               O_g += P_g(j) V_j once P_g(j) is written; a K/V stage is released when both groups' MMAs for that
//               tile are issued.
//   warps 2-5   softmax group 0 (Q tile 0), warps 6-9 group 1 (Q tile 1). Warp w reads TMEM lanes 32*(w%4)..+31.
//
// TMEM columns: [0,KT) S_0, [KT,2KT) S_1, then O_0 and O_1 (D columns each), P_0 and P_1 (KT/2 columns each); the
// softmax warps add the row sums up themselves.
// Every mbarrier wait is bounded (common.cuh): on a timeout all roles stop, in-flight TMA loads and MMAs are waited
// for (bounded), TMEM is freed and the status word records the cause.
#include <algorithm>
#include <cstdlib>
#include <string>
#include <stdexcept>

#include "common.cuh"
#include "launchers.h"

namespace qw {

CUtensorMap make_bf16_map_3d(const void* ptr, int64_t inner, int64_t rows, int64_t batches, int64_t ld,
                             int64_t batch_stride, int box_rows);

namespace attn_fwd_tc {

constexpr int kTile = 128;                    // queries per Q tile
constexpr int kGroups = 2;                    // Q tiles per CTA, one softmax warpgroup each
constexpr int kThreads = 64 + 128 * kGroups;  // TMA warp, MMA warp, softmax warpgroups
constexpr int kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.f;  // move the reference maximum only when a row grows by more than 2^8

template <int D>
struct Layout {
  static constexpr int KT = D == 64 ? 128 : 64;             // keys per K/V tile
  // Row sums on the tensor core (P times a ones row, N = 16) cost as many MMA instructions as P V itself, and an
  // M = 128 MMA instruction takes about the same time at N = 16 as at N = 128; the softmax warps add them up with
  // packed fp32 adds instead. (TMEM would have room for them at head_dim 128.)
  static constexpr bool kRowSumMma = false;
  static constexpr int kStages = D == 64 ? 4 : 3;
  static constexpr int kBoxes = D / 64;                      // 64-wide (128-byte) boxes per row
  static constexpr int kQBytes = kBoxes * kTile * 128;       // one [128 x D] bf16 Q tile
  static constexpr int kKVBytes = kBoxes * KT * 128;         // one [KT x D] bf16 K or V tile
  static constexpr int kQ = 0;
  static constexpr int kKV = kGroups * kQBytes;              // stages of [K | V]
  static constexpr int kOnes = kKV + kStages * 2 * kKVBytes; // [16 x KT] K-major B operand: row 0 ones, rows 1-15 zero
  static constexpr int kOnesBytes = kRowSumMma ? (KT / 64) * 16 * 128 : 0;
  static constexpr int kBar = kOnes + kOnesBytes;
  static constexpr int kTotal = kBar + 256 + 1024;           // barriers, and slack to align the base to 1 KB
  static constexpr int kTmemO = 2 * KT;                      // first column of the partial outputs
  static constexpr int kTmemP = kTmemO + kGroups * D;        // P_g: 128 x KT bf16, two per 32-bit column
  static constexpr int kTmemL = kTmemP + kGroups * (KT / 2); // row sums (head_dim 128), 16 columns per group
  static_assert(kTmemL + (kRowSumMma ? kGroups * 16 : 0) <= kTmemCols, "TMEM columns");
  static_assert(kTotal <= 227 * 1024, "shared memory per CTA");
};

struct Params {
  bf16* o;
  int64_t ldo;
  float* lse;  // [B, Hq, S]
  int S, Hq, Hkv;
  float scale_log2;  // softmax scale * log2(e)
  int park;          // idle MMA issuer: 1 = suspend on a pending P barrier (hinted try_wait), 0 = spin
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Optional timeline of the CTA at blockIdx (0, 0) (clock64 of its SM) for tuning: null unless armed from the host
// (attn_fwd_trace). Slots of (tile j, group g) at 8 * (2j + g): 0 scores ready, 1 probabilities computed,
// 2 previous P V done, 3 P written, 4 S(j) issued, 5 O(j) issued.
constexpr int kTraceTiles = 32;
static __device__ unsigned long long* g_attn_fwd_trace;

__device__ __forceinline__ void trace_mark(unsigned long long* tr, int j, int g, int slot) {
  if (tr && j < kTraceTiles) tr[(2 * j + g) * 8 + slot] = clock64();
}

// K/V tiles of KT keys that the 128 queries from q_start see (causal: keys up to the last query of the tile)
template <int KT>
__device__ __forceinline__ int kv_tiles_of(const Params& p, int q_start) {
  if (q_start >= p.S) return 0;
  return (min(p.S, q_start + kTile) + KT - 1) / KT;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, Params p) {
  using L = Layout<D>;
  constexpr int KT = L::KT;
  constexpr int kStages = L::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* kv_full = q_full + 1;           // [kStages]
  uint64_t* kv_empty = kv_full + kStages;   // [kStages]
  uint64_t* s_full = kv_empty + kStages;    // [kGroups] S_g of the group's next tile is in TMEM
  uint64_t* s_free = s_full + kGroups;      // [kGroups] the group has read S_g out of TMEM
  uint64_t* p_full = s_free + kGroups;      // [kGroups] P_g written (and O_g rescaled if it had to be)
  uint64_t* o_full = p_full + kGroups;      // [kGroups] O_g += P_g V_j has completed
  uint64_t* teardown = o_full + kGroups;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(teardown + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  unsigned long long* const trace = (blockIdx.x == 0 && blockIdx.y == 0) ? g_attn_fwd_trace : nullptr;
  const int b = blockIdx.x / p.Hq, hq = blockIdx.x % p.Hq;
  const int hk = hq / (p.Hq / p.Hkv);
  const int q0 = (gridDim.y - 1 - blockIdx.y) * (kTile * kGroups);  // the latest queries see the most keys: first
  const int n0 = kv_tiles_of<KT>(p, q0), n1 = kv_tiles_of<KT>(p, q0 + kTile);
  const int nk = max(n0, n1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < kGroups; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&s_free[g], 4);  // one arrival per warp of the group
      mbar_init(&p_full[g], 4);
      mbar_init(&o_full[g], 1);
    }
    mbar_init(teardown, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // the ones operand of the row-sum MMA: row 0 of each 64-key box is all ones (the swizzle only permutes 16-byte
  // chunks inside a row, so a row of ones needs none), rows 1-15 are zero
  if constexpr (L::kRowSumMma) {
    for (int i = threadIdx.x; i < L::kOnesBytes / 16; i += kThreads) {
      const uint32_t one = (i % 128) < 8 ? 0x3F803F80u : 0u;
      reinterpret_cast<uint4*>(smem + L::kOnes)[i] = make_uint4(one, one, one, one);
    }
    fence_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // phase of the last load issued into each stage (-1: none), packed 2 bits per stage to stay in a register
      uint32_t issued = 0;  // bit 2s: stage s used, bit 2s+1: its phase
      mbar_arrive_expect_tx(q_full, kGroups * L::kQBytes);
#pragma unroll
      for (int g = 0; g < kGroups; ++g)
#pragma unroll
        for (int c = 0; c < L::kBoxes; ++c)
          tma_load_3d(smem + L::kQ + g * L::kQBytes + c * kTile * 128, &map_q, q_full, hq * D + c * 64,
                      q0 + g * kTile, b);
      for (int j = 0; j < nk; ++j) {
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_sleep_wait(&kv_empty[st], ph ^ 1, kTimeoutEmpty) || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[st], 2 * L::kKVBytes);
        issued = (issued & ~(3u << (2 * st))) | ((1u | (ph << 1)) << (2 * st));
        uint8_t* sk = smem + L::kKV + st * 2 * L::kKVBytes;
#pragma unroll
        for (int c = 0; c < L::kBoxes; ++c) {
          tma_load_3d(sk + c * KT * 128, &map_k, &kv_full[st], hk * D + c * 64, j * KT, b);
          tma_load_3d(sk + L::kKVBytes + c * KT * 128, &map_v, &kv_full[st], hk * D + c * 64, j * KT, b);
        }
      }
      // drain: every load issued above has landed before the CTA may exit
      mbar_sleep_wait(q_full, 0, kTimeoutFull);
      for (int s = 0; s < kStages; ++s)
        if ((issued >> (2 * s)) & 1u) mbar_sleep_wait(&kv_full[s], (issued >> (2 * s + 1)) & 1u, kTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16(kTile, KT, false, false);
      constexpr uint32_t id_o = idesc_bf16(kTile, D, false, true);
      constexpr uint32_t id_l = idesc_bf16(kTile, 16, false, false);
      const uint32_t sones = smem_u32(smem + L::kOnes);
      int ns0 = 0, ns1 = 0;  // next S to issue, per group
      int no0 = 0, no1 = 0;  // next O' to issue, per group
      int released = 0;      // K/V tiles whose stage went back to the producer
      // The issuer shares its SM sub-partition with two softmax warps, so it gets a fraction of the issue slots:
      // every descriptor below is a precomputed base plus a constant (the 14-bit address field holds bytes / 16),
      // leaving about one add and the MMA itself per instruction.
      const uint64_t dq0 = smem_desc_sw128(smem_u32(smem + L::kQ), 16, 1024);
      const uint64_t dk0 = smem_desc_sw128(smem_u32(smem + L::kKV), 16, 1024);
      const uint64_t dv0 = smem_desc_sw128(smem_u32(smem + L::kKV + L::kKVBytes), KT * 128, 1024);
      const uint64_t d1 = smem_desc_sw128(sones, 16, 1024);
      auto issue_s = [&](int g, int j) {
        const uint64_t dq = dq0 + static_cast<uint32_t>(g * (L::kQBytes >> 4));
        const uint64_t dk = dk0 + static_cast<uint32_t>((j % kStages) * ((2 * L::kKVBytes) >> 4));
        const uint32_t d = tmem + g * KT;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k)  // 16 head-dim columns per MMA: 32 bytes inside a 128-byte box
          umma_bf16(d, dq + (((k / 4) * (kTile * 128) + (k % 4) * 32) >> 4), dk + (((k / 4) * (KT * 128) + (k % 4) * 32) >> 4),
                    id_s, k > 0 ? 1u : 0u);
        umma_commit(&s_full[g]);
        trace_mark(trace, j, g, 4);
      };
      auto issue_o = [&](int g, int j) {
        const uint64_t dv = dv0 + static_cast<uint32_t>((j % kStages) * ((2 * L::kKVBytes) >> 4));
        const uint32_t a0 = tmem + L::kTmemP + g * (KT / 2);
        const uint32_t d = tmem + L::kTmemO + g * D;
        const uint32_t first = j > 0 ? 1u : 0u;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < KT / 16; ++k) {
          // A = P_g from TMEM (16 keys = 8 columns per step); B = V read MN-major: 16 keys = 16 rows of 128 B per
          // step, 64-wide head-dim blocks one box (KT rows) apart
          umma_bf16_ts(d, a0 + k * 8, dv + ((k * 2048) >> 4), id_o, k > 0 ? 1u : first);
          if constexpr (L::kRowSumMma)  // l_g += P_g 1: the row sums, from the same A and the K-major ones row
            umma_bf16_ts(tmem + L::kTmemL + g * 16, a0 + k * 8, d1 + ((((k / 4) * (16 * 128) + (k % 4) * 32)) >> 4), id_l,
                         k > 0 ? 1u : first);
        }
        umma_commit(&o_full[g]);
        trace_mark(trace, j, g, 5);
      };
      bool ok = mbar_sleep_wait(q_full, 0, kTimeoutFull);
      tc_fence_after();
      int idle = 0;
      uint64_t idle_start = 0;
      // one group's step: O_g += P_g(j) V_j once the group has written P_g(j); S_g(j) once tile j has landed and
      // the group has read S_g(j-1) out of the TMEM columns this MMA overwrites
      auto step = [&](int g, int n, int& ns, int& no) -> bool {
        bool moved = false;
        if (no < ns && mbar_test(&p_full[g], no & 1)) {
          issue_o(g, no++);
          moved = true;
        }
        if (ns < n && (ns == 0 || mbar_test(&s_free[g], (ns - 1) & 1)) &&
            mbar_test(&kv_full[ns % kStages], (ns / kStages) & 1)) {
          issue_s(g, ns++);
          moved = true;
        }
        return moved;
      };
      while (ok && (no0 < n0 || no1 < n1)) {
        bool progress = step(0, n0, ns0, no0);
        progress = step(1, n1, ns1, no1) || progress;
        while (released < nk && (released >= n0 || no0 > released) && (released >= n1 || no1 > released)) {
          umma_commit(&kv_empty[released % kStages]);  // fires when the MMAs reading that stage are done
          ++released;
          progress = true;
        }
        if (progress) {
          idle = 0;
          continue;
        }
        // nothing ready: by default suspend on a pending P barrier with a short hint (the thread wakes when that
        // barrier completes or the hint runs out), so the idle issuer takes no issue slots from the softmax warps
        // sharing its SM sub-partition; QW_ATTN_ISSUER=spin polls
        if (p.park) {
          if (no0 < ns0) mbar_try_wait_hint(&p_full[0], no0 & 1, 256u);
          else if (no1 < ns1) mbar_try_wait_hint(&p_full[1], no1 & 1, 256u);
        }
        if ((++idle & 1023) == 0) {  // bounded: give up after the wait budget without progress
          if (*abort_flag) { ok = false; break; }
          const uint64_t now = globaltimer();
          if (idle == 1024) idle_start = now;
          else if (now - idle_start > QW_WAIT_TIMEOUT_NS) { set_status(kTimeoutAccum); ok = false; break; }
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(teardown);  // fires once every MMA issued above has completed
      mbar_sleep_wait(teardown, 0, kTimeoutAccum);
    }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups (warps 2..9)
    const int g = (warp - 2) / 4;
    const int quarter = warp % 4;
    const int row = quarter * 32 + lane;
    const int q_start = q0 + g * kTile;
    const int q = q_start + row;
    const int n = g == 0 ? n0 : n1;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t ts = tmem + lane_off + g * KT;
    const uint32_t to = tmem + lane_off + L::kTmemO + g * D;
    const uint32_t tl = tmem + lane_off + L::kTmemL + g * 16;
    const uint32_t tp = tmem + lane_off + L::kTmemP + g * (KT / 2);
    unsigned long long* const gtrace = (quarter == 2 && lane == 0) ? trace : nullptr;
    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY;  // the maximum O_g and l_g are expressed against (base-2, scaled)
    float l_sum = 0.f;        // row sum of the probabilities (head_dim 64; at 128 the tensor core forms it)
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
      if (!__all_sync(0xffffffffu, mbar_sleep_wait(&s_full[g], j & 1, kTimeoutAccum))) { ok = false; break; }
      trace_mark(gtrace, j, g, 0);
      tc_fence_after();
      float v[KT];
#pragma unroll
      for (int c = 0; c < KT; c += 64) tmem_ld32_pair(ts + c, ts + c + 32, v + c, v + c + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[g]);  // the issuer may compute the next scores into these columns
      const int k0 = j * KT;
      // tiles that reach past the group's first query, and a tile past the end of the sequence, need masking; the
      // others (all but one or two per row) take the loop below without any per-key test
      if ((k0 + KT - 1 > q_start) || (k0 + KT > p.S)) {
        const int lim = min(q + 1, p.S) - k0;  // keys [k0, k0 + lim) are visible to this row
#pragma unroll
        for (int i = 0; i < KT; ++i)
          if (i >= lim) v[i] = -INFINITY;
      }
      // row maximum of the raw scores (the scale is positive), three at a time
      float mx = v[0];
#pragma unroll
      for (int i = 1; i + 1 < KT; i += 2) mx = fmax3(mx, v[i], v[i + 1]);
      mx = fmaxf(mx, v[KT - 1]) * sl2;
      // the reference maximum moves only when some row of the warp grew by more than 2^8 (warp-uniform decision:
      // TMEM access is warp-collective); rows whose maximum barely moved then get a factor close to 1
      float factor = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_ref = mx;  // key 0 is visible to every row, so the first tile's maximum is finite
      } else if (__any_sync(0xffffffffu, mx > m_ref + kRescaleLog2)) {
        const float m_new = fmaxf(m_ref, mx);
        factor = ex2(m_ref - m_new);
        m_ref = m_new;
        rescale = true;
      }
      // probabilities, two per instruction in half precision: the exponent s*scale*log2e - m_ref lies in [-inf, 8]
      // thanks to the lazy rescale, so its f16 rounding keeps ~11 bits where the probabilities are large (the bf16
      // probabilities keep 8)
      const float2 scale2 = make_float2(sl2, sl2), neg_m2 = make_float2(-m_ref, -m_ref);
      uint32_t pk[KT / 2];
      float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < KT / 2; ++i) {
        const float2 x = fma_f32x2(make_float2(v[2 * i], v[2 * i + 1]), scale2, neg_m2);
        const float2 e = exp2_f16x2(x.x, x.y);
        pk[i] = pack_bf16(e.x, e.y);  // exp2(-inf) = 0 for masked keys
        if constexpr (!L::kRowSumMma) sum2 = add_f32x2(sum2, e);
      }
      const float tile_sum = sum2.x + sum2.y;
      trace_mark(gtrace, j, g, 1);
      // O_g += P_g(j-1) V_{j-1} must have finished before its P buffer is rewritten or O_g is rescaled
      if (j > 0 && !__all_sync(0xffffffffu, mbar_sleep_wait(&o_full[g], (j - 1) & 1, kTimeoutAccum))) {
        ok = false;
        break;
      }
      trace_mark(gtrace, j, g, 2);
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < KT / 2; c += 32) tmem_st32u(tp + c, pk + c);  // P_g(j): row = lane, key pairs = columns
      if constexpr (!L::kRowSumMma) l_sum = fmaf(l_sum, factor, tile_sum);
      if (rescale) {  // O_g and l_g to the new reference before the next P V accumulates into them
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          float o[32];
          tmem_ld32(to + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= factor;
          tmem_st32(to + c, o);
        }
        if constexpr (L::kRowSumMma) {
          float l[16];
          tmem_ld16(tl, l);
#pragma unroll
          for (int i = 0; i < 16; ++i) l[i] *= factor;
          tmem_st16(tl, l);
        }
      }
      tmem_st_wait();  // P (and the rescaled O) are in TMEM before the issuer may read them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
      trace_mark(gtrace, j, g, 3);
    }
    if (ok && n > 0 && !__all_sync(0xffffffffu, mbar_sleep_wait(&o_full[g], (n - 1) & 1, kTimeoutAccum))) ok = false;
    if (!ok) {
      *abort_flag = 1;
    } else if (n > 0) {
      tc_fence_after();
      if constexpr (L::kRowSumMma) {
        float l[16];
        tmem_ld16(tl, l);  // column 0: the row sum of the probabilities, relative to m_ref
        l_sum = l[0];
      }
      const float inv = 1.f / l_sum;
      bf16* out = p.o + (static_cast<int64_t>(b) * p.S + q) * p.ldo + hq * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(to + c, o);  // warp-collective: every lane loads, only rows inside the sequence store
        if (q < p.S) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_bf16(o[i] * inv, o[i + 1] * inv);
            w.y = pack_bf16(o[i + 2] * inv, o[i + 3] * inv);
            w.z = pack_bf16(o[i + 4] * inv, o[i + 5] * inv);
            w.w = pack_bf16(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4*>(out + c + i) = w;
          }
        }
      }
      if (q < p.S) p.lse[(static_cast<int64_t>(b) * p.Hq + hq) * p.S + q] = (m_ref + __log2f(l_sum)) * kLn2;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int D>
void run(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, bf16* o, int64_t ldo,
         float* lse, int B, int S, int Hq, int Hkv, float scale, cudaStream_t stream) {
  auto kernel = attn_fwd_tc_kernel<D>;
  static bool configured = false;
  if (!configured) {
    check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<D>::kTotal),
               "attention forward tc smem");
    configured = true;
  }
  Params p{};
  p.o = o;
  p.ldo = ldo;
  p.lse = lse;
  p.S = S;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = scale * kLog2e;
  static const int park = [] {
    const char* e = std::getenv("QW_ATTN_ISSUER");
    return (e && std::string(e) == "spin") ? 0 : 1;
  }();
  p.park = park;
  auto mq = make_bf16_map_3d(q, static_cast<int64_t>(Hq) * D, S, B, ldq, S * ldq, kTile);
  auto mk = make_bf16_map_3d(k, static_cast<int64_t>(Hkv) * D, S, B, ldk, S * ldk, Layout<D>::KT);
  auto mv = make_bf16_map_3d(v, static_cast<int64_t>(Hkv) * D, S, B, ldv, S * ldv, Layout<D>::KT);
  dim3 grid(B * Hq, (S + kTile * kGroups - 1) / (kTile * kGroups));
  kernel<<<grid, kThreads, Layout<D>::kTotal, stream>>>(mq, mk, mv, p);
  check_cuda(cudaGetLastError(), "attention forward tc launch");
}

}  // namespace attn_fwd_tc

void flash_attn_fwd_tc(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, bf16* o,
                       int64_t ldo, float* lse, int B, int S, int Hq, int Hkv, int D, float scale,
                       cudaStream_t stream) {
  if (B == 0 || S == 0) return;
  if (D != 64 && D != 128) throw std::runtime_error("flash_attn_fwd_tc: head_dim must be 64 or 128");
  if (Hq % Hkv) throw std::runtime_error("flash_attn_fwd_tc: query heads must be a multiple of kv heads");
  if (D == 64) attn_fwd_tc::run<64>(q, ldq, k, ldk, v, ldv, o, ldo, lse, B, S, Hq, Hkv, scale, stream);
  else attn_fwd_tc::run<128>(q, ldq, k, ldk, v, ldv, o, ldo, lse, B, S, Hq, Hkv, scale, stream);
}

int attention_fwd_tc_status(bool clear) { return read_status_word(clear); }

// Arms (buf: 2 * kTraceTiles * 8 int64 slots) or disarms (null) the forward's timeline trace.
void attn_fwd_trace(void* buf) {
  unsigned long long* ptr = static_cast<unsigned long long*>(buf);
  check_cuda(cudaMemcpyToSymbol(attn_fwd_tc::g_attn_fwd_trace, &ptr, sizeof(ptr)), "attention trace");
}

}  // namespace qw
