// Causal flash-attention backward on the Blackwell tensor cores: tcgen05.mma with TMEM accumulators, operands
// staged by TMA into 128-byte-swizzled shared memory, head_dim 64 or 128, grouped-query attention.
//
// One kernel template serves both passes (deterministic, no atomics):
//
//   dK/dV pass  CTA = 128 keys of one (batch, kv-head). It loops over the group's q-heads and over the 64-query
//               tiles at or after its first key. Row operands X1 = K, X2 = V; column operands Y1 = Q, Y2 = dO.
//                 S^T = K Q^T, dP^T = V dO^T                      (TMEM, 128 x 64, double-buffered)
//                 P^T = exp2(S^T * scale*log2e - lse2[q]),  dS^T = P^T * (dP^T - delta[q])   (softmax warps)
//                 dV += P^T dO,  dK += dS^T Q                    (TMEM, 128 x D each; P^T/dS^T from shared memory)
//   dQ pass     CTA = 128 queries of one (batch, q-head); loops over the 64-key tiles up to the diagonal.
//               X1 = Q, X2 = dO; Y1 = K, Y2 = V.  S = Q K^T, dP = dO V^T, dS = P * (dP - delta[q]), dQ += dS K.
//
// Roles (576 threads, one CTA per SM — the shared-memory request guarantees it, so the 512 TMEM columns never
// contend):
//   warp 0       TMA: the two row tiles once, then the column tiles through a ring of 3 stages; in the dK/dV pass
//                its lanes also stage the 64 lse/delta values of each query tile next to the tile.
//   warp 1       MMA issuer (one thread), polling: S/dP of the next tile as soon as its stage has landed and the
//                softmax group owning its TMEM buffer has loaded that buffer's previous tile, and the accumulation of
//                the oldest tile whose P/dS operands are written — whichever is ready first, so neither the tensor
//                core nor a softmax group waits behind an unrelated condition.
//   warps 2-17   softmax, two groups of 8 warps working on alternate tiles (group g: tiles j % 2 == g, TMEM S/dP
//                buffer g, operand buffer g), so one group's latency chain overlaps the other's. In a group, warp w
//                reads TMEM lanes 32*(w%4).. (its row quarter), and the first four warps take columns 0-31, the last
//                four 32-63. They write bf16 P/dS rows into the swizzled K-major layout the next MMA reads, and at
//                the end read dK/dV (or dQ) out of TMEM and store them.
//
// TMEM columns: [0,128) S (2 x 64), [128,256) dP (2 x 64), [256,256+D) dV or dQ, [256+D,256+2D) dK.
// Every mbarrier wait is bounded (common.cuh): on a timeout all roles stop, in-flight TMA loads and MMAs are
// waited for (bounded), TMEM is freed and the status word records the cause.
#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launchers.h"

namespace qw {

CUtensorMap make_bf16_map_3d(const void* ptr, int64_t inner, int64_t rows, int64_t batches, int64_t ld,
                             int64_t batch_stride, int box_rows);

namespace attn_tc {

constexpr int kRows = 128;                 // tile rows (keys in dK/dV, queries in dQ)
constexpr int kCols = 64;                  // columns per inner step
constexpr int kSoftWarps = 16;  // two groups of 8
constexpr int kThreads = 64 + 32 * kSoftWarps;
constexpr int kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

enum Mode : int { kDKDV = 0, kDQ = 1 };

template <int D, int MODE>
struct Layout {
  static constexpr int kBoxes = D / 64;                      // 64-wide (128-byte) boxes per row
  static constexpr int kXBytes = kBoxes * kRows * 128;       // one row operand
  static constexpr int kYBytes = kBoxes * kCols * 128;       // one column operand
  // tiles j, j+1, j+2 (S issued ahead) resident, plus one stage of TMA lead where shared memory allows
  static constexpr int kStages = (D == 64) ? 6 : 3;
  static constexpr int kOBytes = kRows * kCols * 2;          // one bf16 [128 x 64] operand (P^T or dS)
  static constexpr int kONum = (MODE == kDKDV) ? 2 : 1;
  static constexpr int kX1 = 0;
  static constexpr int kX2 = kXBytes;
  static constexpr int kY = 2 * kXBytes;                     // stages of [Y1 | Y2]
  static constexpr int kO = kY + kStages * 2 * kYBytes;      // 2 buffers of kONum operands
  static constexpr int kVec = kO + 2 * kONum * kOBytes;      // stages of [lse2 | delta] (64 floats each)
  static constexpr int kBar = kVec + kStages * 2 * kCols * 4;
  static constexpr int kUsed = kBar + 256;
  static constexpr int kTotal = (kUsed + 1024 > 120 * 1024) ? kUsed + 1024 : 120 * 1024;
};

struct Params {
  const float* lse;    // [B, Hq, S], natural log
  const float* delta;  // [B, Hq, S]
  bf16* out1;          // dV (dK/dV pass) or dQ
  int64_t ld1;
  bf16* out2;          // dK
  int64_t ld2;
  int S, Hq, Hkv;
  float scale;
  int park;  // idle MMA issuer: 1 = suspend on the oldest pending P/dS barrier (hinted try_wait), 0 = spin
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Optional timeline of CTA (0, 0) (clock64 of its SM) for tuning: null unless armed from the host (attn_bwd_trace).
// Slots of tile t of pass m (0 dK/dV, 1 dQ) at 16 * (32 m + t): 0 S/dP issued, 1 scores ready (softmax), 2 P/dS
// written (first warp of the group), 3 accumulation issued, 4 + w P/dS written by warp w of the group.
constexpr int kTraceTiles = 32;
static __device__ unsigned long long* g_attn_bwd_trace;

template <int MODE>
__device__ __forceinline__ void trace_mark(unsigned long long* tr, int t, int slot) {
  if (tr && t < kTraceTiles) tr[16 * (MODE * kTraceTiles + t) + slot] = clock64();
}

__device__ __forceinline__ void store_row16(bf16* dst, const float* v, float mul) {
#pragma unroll
  for (int i = 0; i < 16; i += 8) {
    uint4 w;
    w.x = pack_bf16(v[i] * mul, v[i + 1] * mul);
    w.y = pack_bf16(v[i + 2] * mul, v[i + 3] * mul);
    w.z = pack_bf16(v[i + 4] * mul, v[i + 5] * mul);
    w.w = pack_bf16(v[i + 6] * mul, v[i + 7] * mul);
    *reinterpret_cast<uint4*>(dst + i) = w;
  }
}

template <int D, int MODE>
// 18 warps: the register file is split over the 4 SM sub-partitions, one of which holds 5 warps, so a thread gets
// at most 16384 / 160 -> 96 registers; __launch_bounds__ lets ptxas apply that limit.
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_do,
                       Params p) {
  using L = Layout<D, MODE>;
  constexpr int kStages = L::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* empty = full + kStages;
  uint64_t* s_full = empty + kStages;  // [2] S/dP of a tile are in TMEM
  uint64_t* s_empty = s_full + 2;      // [2] softmax has read them
  uint64_t* p_full = s_empty + 2;      // [2] P/dS operands written
  uint64_t* p_empty = p_full + 2;      // [2] accumulation MMAs done with them
  uint64_t* x_full = p_empty + 2;
  uint64_t* acc_full = x_full + 1;
  uint64_t* teardown = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(teardown + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  unsigned long long* const trace = (blockIdx.x == 0 && blockIdx.y == 0) ? g_attn_bwd_trace : nullptr;
  const int group = p.Hq / p.Hkv;
  int b, hk, hq, row0, n, per_head;
  if (MODE == kDKDV) {
    b = blockIdx.x / p.Hkv;
    hk = blockIdx.x % p.Hkv;
    hq = hk * group;
    row0 = blockIdx.y * kRows;  // tile 0 (first keys) sees the most queries: scheduled first
    per_head = (p.S - row0 + kCols - 1) / kCols;
    n = per_head * group;
  } else {
    b = blockIdx.x / p.Hq;
    hq = blockIdx.x % p.Hq;
    hk = hq / group;
    row0 = (gridDim.y - 1 - blockIdx.y) * kRows;  // the last query tile sees the most keys: scheduled first
    n = (min(p.S, row0 + kRows) + kCols - 1) / kCols;
    per_head = n;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], MODE == kDKDV ? 2 : 1);  // dK/dV: the TMA arrival plus the lse/delta staging arrival
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kSoftWarps / 2);
      mbar_init(&p_full[i], kSoftWarps / 2);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(x_full, 1);
    mbar_init(acc_full, 1);
    mbar_init(teardown, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
    tma_prefetch_desc(&map_do);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    const CUtensorMap* mx1 = MODE == kDKDV ? &map_k : &map_q;
    const CUtensorMap* mx2 = MODE == kDKDV ? &map_v : &map_do;
    const CUtensorMap* my1 = MODE == kDKDV ? &map_q : &map_k;
    const CUtensorMap* my2 = MODE == kDKDV ? &map_do : &map_v;
    const int xh = MODE == kDKDV ? hk : hq;
    int issued[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) issued[s] = -1;
    if (lane == 0) {
      mbar_arrive_expect_tx(x_full, 2 * L::kXBytes);
#pragma unroll
      for (int c = 0; c < L::kBoxes; ++c) {
        tma_load_3d(smem + L::kX1 + c * kRows * 128, mx1, x_full, xh * D + c * 64, row0, b);
        tma_load_3d(smem + L::kX2 + c * kRows * 128, mx2, x_full, xh * D + c * 64, row0, b);
      }
    }
    // lse2 / delta of the 64 queries of a dK/dV tile: lane l holds columns l and l+32
    float next_l[kCols / 32], next_d[kCols / 32];
    auto load_vec = [&](int t) {
      const int th = hq + t / per_head;
      const int tcs = row0 + (t % per_head) * kCols;
      const int64_t base = (static_cast<int64_t>(b) * p.Hq + th) * p.S;
#pragma unroll
      for (int k = 0; k < kCols / 32; ++k) {
        const int qi = tcs + lane + 32 * k;
        next_l[k] = qi < p.S ? p.lse[base + qi] * kLog2e : 0.f;
        next_d[k] = qi < p.S ? p.delta[base + qi] : 0.f;
      }
    };
    if (MODE == kDKDV && n > 0) load_vec(0);
    int stage = 0;
    uint32_t phase = 0;
    for (int j = 0; j < n; ++j) {
      int go = 1;
      if (lane == 0) go = (mbar_sleep_wait(&empty[stage], phase ^ 1, kTimeoutEmpty) && !*abort_flag) ? 1 : 0;
      go = __shfl_sync(0xffffffffu, go, 0);  // one decision for the whole warp
      if (!go) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      const int yh = MODE == kDKDV ? hq + j / per_head : hk;
      const int cs = MODE == kDKDV ? row0 + (j % per_head) * kCols : j * kCols;
      if (lane == 0) {  // the tile loads first, so their latency overlaps the lse/delta staging below
        mbar_arrive_expect_tx(&full[stage], 2 * L::kYBytes);
        issued[stage] = static_cast<int>(phase);
        uint8_t* y1 = smem + L::kY + stage * 2 * L::kYBytes;
        uint8_t* y2 = y1 + L::kYBytes;
#pragma unroll
        for (int c = 0; c < L::kBoxes; ++c) {
          tma_load_3d(y1 + c * kCols * 128, my1, &full[stage], yh * D + c * 64, cs, b);
          tma_load_3d(y2 + c * kCols * 128, my2, &full[stage], yh * D + c * 64, cs, b);
        }
      }
      if (MODE == kDKDV) {
        // the values of tile j were loaded into registers one iteration earlier; load tile j+1's now, so the
        // global-load latency overlaps this warp's wait for the next free stage instead of serialising the ring
        float* vec = reinterpret_cast<float*>(smem + L::kVec + stage * 2 * kCols * 4);
#pragma unroll
        for (int k = 0; k < kCols / 32; ++k) {
          vec[lane + 32 * k] = next_l[k];
          vec[kCols + lane + 32 * k] = next_d[k];
        }
        if (j + 1 < n) load_vec(j + 1);
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[stage]);  // second arrival: the staged values are written
      }
      if (++stage == kStages) { stage = 0; phase ^= 1; }
    }
    if (lane == 0) {  // drain: every load this warp issued has landed before the CTA may exit
      mbar_sleep_wait(x_full, 0, kTimeoutFull);
      for (int s = 0; s < kStages; ++s)
        if (issued[s] >= 0) mbar_sleep_wait(&full[s], static_cast<uint32_t>(issued[s]), kTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16(kRows, kCols, false, false);
      constexpr uint32_t id_acc = idesc_bf16(kRows, D, false, true);
      const uint32_t sx1 = smem_u32(smem + L::kX1), sx2 = smem_u32(smem + L::kX2);
      // S/dP of tile t into TMEM buffer t&1 (its stage has landed; from t = 2 on, the softmax group owning the buffer
      // has loaded tile t-2)
      auto s_ready = [&](int t) {
        return mbar_test(&full[t % kStages], (t / kStages) & 1) &&
               (t < 2 || mbar_test(&s_empty[t & 1], ((t >> 1) - 1) & 1));
      };
      // The issuer shares its SM sub-partition with four softmax warps, so it gets a fraction of the issue slots:
      // every descriptor below is a precomputed base plus a constant (the 14-bit address field holds bytes / 16),
      // leaving about one add and the MMA itself per instruction.
      const uint64_t dx1 = smem_desc_sw128(sx1, 16, 1024), dx2 = smem_desc_sw128(sx2, 16, 1024);
      const uint64_t dy0 = smem_desc_sw128(smem_u32(smem + L::kY), 16, 1024);             // stage 0 Y1, K-major
      const uint64_t dyt0 = smem_desc_sw128(smem_u32(smem + L::kY), kCols * 128, 1024);  // stage 0 Y1, MN-major
      const uint64_t do0 = smem_desc_sw128(smem_u32(smem + L::kO), 16, 1024);
      constexpr uint32_t kY2 = L::kYBytes >> 4;
      auto issue_s = [&](int t) {
        const int buf = t & 1;
        const uint32_t ys = static_cast<uint32_t>((t % kStages) * ((2 * L::kYBytes) >> 4));
        const uint32_t ts = tmem + buf * kCols, tdp = tmem + 128 + buf * kCols;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t ox = ((k / 4) * (kRows * 128) + (k % 4) * 32) >> 4;
          const uint32_t oy = ((k / 4) * (kCols * 128) + (k % 4) * 32) >> 4;
          umma_bf16(ts, dx1 + ox, dy0 + ys + oy, id_s, k > 0 ? 1u : 0u);
          umma_bf16(tdp, dx2 + ox, dy0 + ys + kY2 + oy, id_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[buf]);
        trace_mark<MODE>(trace, t, 0);
      };
      // accumulation of tile j once the softmax group has written its P/dS operands
      auto issue_acc = [&](int j) {
        const int buf = j & 1;
        const int st = j % kStages;
        const uint64_t b1 = dyt0 + static_cast<uint32_t>(st * ((2 * L::kYBytes) >> 4)), b2 = b1 + kY2;
        const uint64_t a0 = do0 + static_cast<uint32_t>(buf * ((L::kONum * L::kOBytes) >> 4));
        const uint32_t first = j > 0 ? 1u : 0u;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kCols / 16; ++k) {
          const uint32_t acc = k > 0 ? 1u : first;
          // B operands are the column tiles read MN-major: 64-wide MN blocks one box apart, K rows of 128 B
          const uint32_t ob = (k * 2048) >> 4, oa = (k * 32) >> 4;
          if (MODE == kDKDV) {
            umma_bf16(tmem + 256, a0 + oa, b2 + ob, id_acc, acc);                               // dV
            umma_bf16(tmem + 256 + D, a0 + (L::kOBytes >> 4) + oa, b1 + ob, id_acc, acc);       // dK
          } else {
            umma_bf16(tmem + 256, a0 + oa, b1 + ob, id_acc, acc);  // dQ
          }
        }
        umma_commit(&empty[st]);
        umma_commit(&p_empty[buf]);
        trace_mark<MODE>(trace, j, 3);
      };
      bool ok = mbar_sleep_wait(x_full, 0, kTimeoutFull);
      tc_fence_after();
      // issue whichever of (next accumulation, next S/dP) is ready, so neither waits behind the other
      int ns = 0, na = 0;
      int idle = 0;
      uint64_t idle_start = 0;
      while (ok && na < n) {
        bool progress = false;
        if (na < ns && mbar_test(&p_full[na & 1], (na >> 1) & 1)) {
          issue_acc(na++);
          progress = true;
        }
        if (ns < n && s_ready(ns)) {
          issue_s(ns++);
          progress = true;
        }
        if (progress) {
          idle = 0;
          continue;
        }
        // nothing ready: by default suspend on the oldest tile's P/dS barrier with a short hint (the thread wakes
        // when that barrier completes or the hint runs out, then polls both conditions again), so the idle issuer
        // takes no issue slots from the softmax warps sharing its SM sub-partition; QW_ATTN_ISSUER=spin polls
        if (p.park && na < ns) mbar_try_wait_hint(&p_full[na & 1], (na >> 1) & 1, 256u);
        if ((++idle & 1023) == 0) {  // bounded: give up after the wait budget without progress
          if (*abort_flag) { ok = false; break; }
          const uint64_t now = globaltimer();
          if (idle == 1024) idle_start = now;
          else if (now - idle_start > QW_WAIT_TIMEOUT_NS) { set_status(kTimeoutAccum); ok = false; break; }
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(acc_full);  // fires once every MMA issued above has completed
      umma_commit(teardown);
      mbar_sleep_wait(teardown, 0, kTimeoutAccum);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (warps 2..17)
    // group g (warps 2+8g .. 9+8g) takes the tiles j with j % 2 == g and owns TMEM S/dP buffer g and operand buffer g,
    // so the two groups work on consecutive tiles at the same time
    const int sw = warp - 2;
    const int grp = sw / 8;
    const int quarter = warp % 4;
    const int half = (sw % 8) / 4;
    const int row = quarter * 32 + lane;
    const int grow = row0 + row;  // key (dK/dV) or query (dQ) index of this thread's row
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    float row_lse2 = 0.f, row_delta = 0.f;
    if (MODE == kDQ && grow < p.S) {
      const int64_t idx = (static_cast<int64_t>(b) * p.Hq + hq) * p.S + grow;
      row_lse2 = p.lse[idx] * kLog2e;
      row_delta = p.delta[idx];
    }
    bool ok = true;
    for (int j = grp; j < n; j += 2) {
      // every exit decision is warp-uniform: the TMEM loads and __syncwarp below need the full warp
      if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
      const int buf = grp;
      const uint32_t use = (j >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_sleep_wait(&s_full[buf], use, kTimeoutAccum))) { *abort_flag = 1; ok = false; break; }
      if (sw % 8 == 0 && lane == 0) trace_mark<MODE>(trace, j, 1);
      tc_fence_after();
      float s[32], dp[32];
      tmem_ld32_pair(tmem + lane_off + buf * kCols + half * 32, tmem + lane_off + 128 + buf * kCols + half * 32, s, dp);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[buf]);

      const int cs = MODE == kDKDV ? row0 + (j % per_head) * kCols : j * kCols;
      const int col0 = cs + half * 32;
      bool need_mask = (col0 + 32 > p.S) || (row0 + kRows > p.S);
      if (MODE == kDKDV) need_mask = need_mask || (col0 < row0 + kRows);
      else need_mask = need_mask || (col0 + 31 > row0);
      const float* vec = nullptr;
      if (MODE == kDKDV) {
        const int st = j % kStages;
        if (!__all_sync(0xffffffffu, mbar_sleep_wait(&full[st], (j / kStages) & 1, kTimeoutFull))) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        vec = reinterpret_cast<const float*>(smem + L::kVec + st * 2 * kCols * 4) + half * 32;
      }
      if (!__all_sync(0xffffffffu, mbar_sleep_wait(&p_empty[buf], use ^ 1, kTimeoutAccumFree))) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      uint8_t* obuf = smem + L::kO + buf * L::kONum * L::kOBytes + row * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // 8 columns -> one 16-byte chunk of P and of dS
        uint32_t pw[4], dw[4];
        float lv[8], dv[8];  // lse2 / delta of the chunk's 8 columns (broadcast 16-byte shared loads)
        if (MODE == kDKDV) {
          const float4* v4 = reinterpret_cast<const float4*>(vec) + 2 * q;
          const float4 l0 = v4[0], l1 = v4[1], d0 = v4[kCols / 4], d1 = v4[kCols / 4 + 1];
          lv[0] = l0.x; lv[1] = l0.y; lv[2] = l0.z; lv[3] = l0.w; lv[4] = l1.x; lv[5] = l1.y; lv[6] = l1.z; lv[7] = l1.w;
          dv[0] = d0.x; dv[1] = d0.y; dv[2] = d0.z; dv[3] = d0.w; dv[4] = d1.x; dv[5] = d1.y; dv[6] = d1.z; dv[7] = d1.w;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) { lv[e] = row_lse2; dv[e] = row_delta; }
        }
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {  // column pairs: packed fp32x2 math, one f16x2 exponential per pair (the
                                          // exponent s*scale*log2e - lse is <= 0 here: P <= 1, and its f16
                                          // rounding keeps ~11 bits where P is large; P and dS go out in bf16)
          const int e = 2 * e2, c = 8 * q + e;
          const float2 arg = fma_f32x2(make_float2(s[c], s[c + 1]), make_float2(sl2, sl2),
                                       make_float2(-lv[e], -lv[e + 1]));
          float2 x = exp2_f16x2(arg.x, arg.y);
          if (need_mask) {
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int other = col0 + c + h2;  // query (dK/dV) or key (dQ) index of this column
              const bool bad = MODE == kDKDV ? (other < grow || other >= p.S || grow >= p.S)
                                             : (other > grow || other >= p.S || grow >= p.S);
              if (bad) (h2 ? x.y : x.x) = 0.f;
            }
          }
          const float2 ds = mul_f32x2(x, add_f32x2(make_float2(dp[c], dp[c + 1]), make_float2(-dv[e], -dv[e + 1])));
          pw[e2] = pack_bf16(x.x, x.y);
          dw[e2] = pack_bf16(ds.x, ds.y);
        }
        const int chunk = (half * 4 + q) ^ (row & 7);
        if (MODE == kDKDV) {
          *reinterpret_cast<uint4*>(obuf + chunk * 16) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
          *reinterpret_cast<uint4*>(obuf + L::kOBytes + chunk * 16) = make_uint4(dw[0], dw[1], dw[2], dw[3]);
        } else {
          *reinterpret_cast<uint4*>(obuf + chunk * 16) = make_uint4(dw[0], dw[1], dw[2], dw[3]);
        }
      }
      fence_async_smem();  // generic-proxy stores -> visible to the tensor core's async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[buf]);
      if (sw % 8 == 0 && lane == 0) trace_mark<MODE>(trace, j, 2);
      if (lane == 0) trace_mark<MODE>(trace, j, 4 + sw % 8);
    }
    // epilogue: accumulators -> bf16 rows (dK and dQ carry the softmax scale). dK/dV: group 0 stores dV, group 1
    // dK, each half of the columns; dQ: each (group, half) a quarter of the columns.
    if (__all_sync(0xffffffffu, ok && !*abort_flag)) {
      if (__all_sync(0xffffffffu, mbar_sleep_wait(acc_full, 0, kTimeoutAccum))) {
        tc_fence_after();
        const int64_t tok = static_cast<int64_t>(b) * p.S + grow;
        int c0, c1, tcol;
        bf16* out;
        float mul;
        if (MODE == kDKDV) {
          c0 = half * (D / 2);
          c1 = c0 + D / 2;
          tcol = 256 + grp * D;
          out = grp == 0 ? p.out1 + tok * p.ld1 + hk * D : p.out2 + tok * p.ld2 + hk * D;
          mul = grp == 0 ? 1.f : p.scale;
        } else {
          c0 = (2 * grp + half) * (D / 4);
          c1 = c0 + D / 4;
          tcol = 256;
          out = p.out1 + tok * p.ld1 + hq * D;
          mul = p.scale;
        }
        for (int c = c0; c < c1; c += 16) {
          float v[16];
          tmem_ld16(tmem + lane_off + tcol + c, v);
          if (grow < p.S) store_row16(out + c, v, mul);
        }
      } else {
        *abort_flag = 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int D, int MODE>
void launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
            const Params& p, dim3 grid, cudaStream_t stream) {
  auto kernel = attn_bwd_tc_kernel<D, MODE>;
  static bool configured = false;
  if (!configured) {
    check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<D, MODE>::kTotal),
               "attention tc smem");
    configured = true;
  }
  kernel<<<grid, kThreads, Layout<D, MODE>::kTotal, stream>>>(mq, mk, mv, mdo, p);
  check_cuda(cudaGetLastError(), "attention tc launch");
}

template <int D>
void run(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv, const bf16* dout,
         int64_t lddo, const float* lse, const float* delta, bf16* dq, int64_t lddq, bf16* dk, int64_t lddk, bf16* dv,
         int64_t lddv, int B, int S, int Hq, int Hkv, float scale, cudaStream_t stream) {
  const int tiles = (S + kRows - 1) / kRows;
  Params p{};
  p.lse = lse;
  p.delta = delta;
  p.S = S;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = scale;
  static const int park = [] {
    const char* e = std::getenv("QW_ATTN_ISSUER");
    return (e && std::string(e) == "spin") ? 0 : 1;
  }();
  p.park = park;
  // dK/dV: K, V are 128-row tiles; Q, dO 64-row tiles
  {
    auto mq = make_bf16_map_3d(q, static_cast<int64_t>(Hq) * D, S, B, ldq, S * ldq, kCols);
    auto mdo = make_bf16_map_3d(dout, static_cast<int64_t>(Hq) * D, S, B, lddo, S * lddo, kCols);
    auto mk = make_bf16_map_3d(k, static_cast<int64_t>(Hkv) * D, S, B, ldk, S * ldk, kRows);
    auto mv = make_bf16_map_3d(v, static_cast<int64_t>(Hkv) * D, S, B, ldv, S * ldv, kRows);
    p.out1 = dv;
    p.ld1 = lddv;
    p.out2 = dk;
    p.ld2 = lddk;
    launch<D, kDKDV>(mq, mk, mv, mdo, p, dim3(B * Hkv, tiles), stream);
  }
  // dQ: Q, dO are 128-row tiles; K, V 64-row tiles
  {
    auto mq = make_bf16_map_3d(q, static_cast<int64_t>(Hq) * D, S, B, ldq, S * ldq, kRows);
    auto mdo = make_bf16_map_3d(dout, static_cast<int64_t>(Hq) * D, S, B, lddo, S * lddo, kRows);
    auto mk = make_bf16_map_3d(k, static_cast<int64_t>(Hkv) * D, S, B, ldk, S * ldk, kCols);
    auto mv = make_bf16_map_3d(v, static_cast<int64_t>(Hkv) * D, S, B, ldv, S * ldv, kCols);
    p.out1 = dq;
    p.ld1 = lddq;
    p.out2 = nullptr;
    p.ld2 = 0;
    launch<D, kDQ>(mq, mk, mv, mdo, p, dim3(B * Hq, tiles), stream);
  }
}

}  // namespace attn_tc

void flash_attn_bwd_tc(const bf16* q, int64_t ldq, const bf16* k, int64_t ldk, const bf16* v, int64_t ldv,
                       const bf16* dout, int64_t lddo, const float* lse, const float* delta, bf16* dq, int64_t lddq,
                       bf16* dk, int64_t lddk, bf16* dv, int64_t lddv, int B, int S, int Hq, int Hkv, int D,
                       float scale, cudaStream_t stream) {
  if (B == 0 || S == 0) return;
  if (D == 64)
    attn_tc::run<64>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dq, lddq, dk, lddk, dv, lddv, B, S, Hq, Hkv, scale,
                     stream);
  else if (D == 128)
    attn_tc::run<128>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dq, lddq, dk, lddk, dv, lddv, B, S, Hq, Hkv,
                      scale, stream);
  else
    throw std::runtime_error("flash_attn_bwd_tc: head_dim must be 64 or 128");
}

int attention_tc_status(bool clear) { return read_status_word(clear); }

// Arms (buf: 2 * 16 * kTraceTiles int64 slots) or disarms (null) the backward's timeline trace.
void attn_bwd_trace(void* buf) {
  unsigned long long* ptr = static_cast<unsigned long long*>(buf);
  check_cuda(cudaMemcpyToSymbol(attn_tc::g_attn_bwd_trace, &ptr, sizeof(ptr)), "attention backward trace");
}

}  // namespace qw
