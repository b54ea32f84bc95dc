// Persistent, warp-specialised tcgen05 GEMM for sm_100a (bf16 in, fp32 accumulate in TMEM).
//
//   C[m, n] = sum_k A[m, k] * B[n, k]        (A: M x K, B: N x K, either operand K-major or MN-major in memory)
//
// Roles (192 threads = 6 warps, one CTA per SM):
//   warp 0     TMA producer: one elected thread streams A/B k-blocks (64 wide, 128-byte swizzle) into a ring of
//              shared-memory stages, signalling `full[s]` with the transaction byte count.
//   warp 1     MMA issuer: allocates 2 x BN TMEM columns (double-buffered accumulators), one thread issues
//              tcgen05.mma (M=128, N=BN, K=16) and frees each stage with tcgen05.commit -> `empty[s]`; after the
//              last k-block of a tile it commits `accum_full[b]`.
//   warps 2-5  epilogue: tcgen05.ld the 128 x BN accumulator (warp w owns TMEM lanes 32*(w%4)..+31 = tile rows),
//              apply the fused epilogue and store to global memory, then release the buffer (`accum_empty[b]`).
//              bf16 outputs go through a per-warp shared-memory box: each lane writes its row, then the warp
//              stores 4 whole 128-byte rows per instruction (a residual comes in the same way). One thread per row
//              storing 16 bytes to 32 different rows per instruction left the epilogue at ~2.5x the k-loop time of
//              a K = 1024 tile. fp32 outputs, read-modify-write accumulation and stores into peers' memory keep the
//              per-thread path.
//
// Tile schedules (device-side, no host synchronisation):
//   kGroupM  grouped over rows: group g owns rows [row_off[g], row_off[g]+rows[g]) of A and C, and its own B
//            (B row base g*b_group_rows). Forward expert GEMMs and their input gradients.
//   kGroupK  grouped over the reduction: group g reduces over rows [row_off[g], ...+rows[g]) of both operands and
//            writes its own C block (C + g*c_group_stride). Weight gradients (dW = dY^T X per expert).
// Grouped row segments are padded to 128 rows with zero rows, so a tile never mixes two groups.
//
// Every mbarrier wait is bounded (see common.cuh); on a timeout all roles stop, in-flight TMA loads are drained
// with a bounded wait, TMEM is freed and the kernel returns with qw_status set.
#pragma once

#include "common.cuh"

namespace qw {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;

enum Mode : int { kGroupM = 0, kGroupK = 1 };

enum Epi : int {
  kEpiStore = 0,      // C = alpha*acc (+bias[n]) (+residual[m,n]) (+C if accumulate); bf16 or fp32 out
  kEpiSwiGLU = 1,     // acc = [gate(BN/2) | up(BN/2)] -> H = silu(g)*u ; optional raw GU store
  kEpiSwiGLUBwd = 2,  // acc = dH (unweighted) ; reads GU, route weight w ; writes dGU, w*H, per-row <acc,H> partials
};

struct Params {
  int M, N, K;                 // dense sizes (kGroupM: M unused; kGroupK: K unused)
  int num_groups;
  const int* group_rows;       // rows per group (kGroupM: M_g ; kGroupK: K_g)
  const int* group_off;        // padded first row of each group
  int b_group_rows;            // kGroupM: B row/K offset between groups
  int expert_mod;              // >0: group g uses B block (g % expert_mod) (groups = (source, local expert) pairs)
  int k_segments;              // kGroupK: each group reduces over this many row segments; segment s of group g uses
                               // group_rows/group_off entry s*num_groups + g (1 = a single contiguous segment)
  int dual_b_offset;           // >0: second half of each N tile comes from B rows + dual_b_offset (gate | up)
  int n_tiles;                 // ceil(N / BN) (kEpiSwiGLU: ceil(F / (BN/2)))
  int m_tiles;                 // kGroupK: ceil(M / 128)
  int max_tiles;               // upper bound used when group sizes are device-side
  int k_chunk;                 // kGroupK without group_rows: group g reduces rows [g*k_chunk, min(K, (g+1)*k_chunk))
                               // and writes its own C block (split-K with per-chunk partial outputs)
  // epilogue
  void* out;
  long ldo;
  long out_group_stride;       // kGroupK: elements between group outputs
  // fused tensor-parallel reduction (kGroupM, bf16): output row m belongs to rank m / peer_rows and is stored over
  // NVLink into that rank's staging buffer peer_out[owner] at row peer_slot * peer_rows + m % peer_rows
  void* const* peer_out;
  long peer_rows;
  int peer_slot;
  int out_fp32;
  int accumulate;
  float alpha;
  const float* bias;
  const __nv_bfloat16* residual;
  long ldr;
  int zero_pad_rows;           // write zeros into padded rows of a group's last tile
  // SwiGLU
  int ffn;                     // F
  __nv_bfloat16* gu_out;       // kEpiSwiGLU: optional raw [gate|up] store, ld = 2F
  const __nv_bfloat16* gu_in;  // kEpiSwiGLUBwd: saved/recomputed [gate|up], ld = 2F
  const float* route_w;        // kEpiSwiGLUBwd: per-row route weight
  __nv_bfloat16* h_out;        // kEpiSwiGLUBwd: optional H = silu(g)*u, ld = F
  float* dw_partial;           // kEpiSwiGLUBwd: [rows, n_tiles] partial <dH_raw, H>
  int staged_out;              // store / SwiGLU epilogues: out through a shared-memory box, coalesced stores
  int tma_out;                 // kGroupM store / SwiGLU, bf16: out (and residual, gu) through TMA boxes instead
};

constexpr int kStgBytes = 32 * 128;  // one epilogue warp's staging box: 32 rows x 64 bf16 (128-byte rows)

template <int BN>
struct Smem {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kDataBytes = kStages * kStageBytes;
  static constexpr int kStg = kDataBytes;                    // 4 epilogue warps x one box each
  static constexpr int kBarOff = kStg + 4 * kStgBytes;
  static constexpr int kTotal = kBarOff + 1024 /*align*/ + 256 /*barriers*/;
};

// TMA stores from shared memory (bulk async-groups of the issuing thread)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               :: "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y) : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One epilogue warp's staging box: 64 bf16 of row `lane` in 16-byte chunks at the 128-byte-swizzled positions the
// tensor map expects (chunk q of row r at q ^ (r % 8); the box is 1024-byte aligned).
struct StageBox {
  uint8_t* base;
  int lane;
  __device__ __forceinline__ uint4* chunk(int q) const {
    return reinterpret_cast<uint4*>(base + lane * 128 + ((q ^ (lane & 7)) << 4));
  }
};

// Per-warp state of the TMA epilogue: the staging box, the maps and the residual barrier's phase.
struct TmaEpi {
  StageBox box;
  const CUtensorMap* map_out;
  const CUtensorMap* map_res;
  const CUtensorMap* map_gu;
  uint64_t* res_bar;
  uint32_t res_phase;
  int row;  // first output row of this warp's 32 rows
};

// Make the warp's box free for new data (the previous bulk store from it has finished reading it).
__device__ __forceinline__ void box_acquire(int lane) {
  if (lane == 0) tma_store_wait_read();
  __syncwarp();
}

// Publish the box written by the warp's lanes and store it at (x, row) through `map`.
__device__ __forceinline__ void box_release(const TmaEpi& e, const CUtensorMap* map, int x, int lane) {
  fence_async_smem();  // generic-proxy writes -> visible to the TMA (async proxy)
  __syncwarp();
  if (lane == 0) tma_store_2d(map, e.box.base, x, e.row);
}

// Staged epilogue of one warp: its 32 rows x 64 columns pass through a shared-memory box so that global memory sees
// whole 128-byte lines. Lane r owns accumulator row r and writes it into the box (16-byte chunk q at q ^ (r % 8),
// so the 32 lanes' chunks fall on distinct banks); then lane l moves chunk l % 8 of rows l / 8 + 4i, i < 8: one
// 16-byte load or store instruction covers 4 full rows.
struct StagedEpi {
  uint8_t* box;  // 4 KB
  int lane;
  long out_rows;  // rows of the output that exist (dense tail); grouped tiles write their padded rows
  __device__ __forceinline__ uint4* own(int q) const {  // chunk q of the lane's own row
    return reinterpret_cast<uint4*>(box + lane * 128 + ((q ^ (lane & 7)) << 4));
  }
  __device__ __forceinline__ uint4* moved(int i) const {  // the chunk this lane moves in step i
    const int r = lane / 8 + 4 * i;
    return reinterpret_cast<uint4*>(box + r * 128 + (((lane & 7) ^ (r & 7)) << 4));
  }
  __device__ __forceinline__ void put(const float* v) const {  // 64 values of the lane's row, rounded to bf16
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *own(q) = make_uint4(pack_bf16(v[8 * q], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                           pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7]));
  }
  __device__ __forceinline__ void put_f32(const float* v) const {  // 32 fp32 values of the lane's row
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *own(q) = make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]), __float_as_uint(v[4 * q + 2]),
                           __float_as_uint(v[4 * q + 3]));
  }
  // box -> 128 bytes at out + (row0 + r) * ld_bytes + col_bytes for rows below out_rows; chunks at or past
  // lim_bytes (the end of the row) are skipped. fp32_add: add the existing fp32 values (read-modify-write).
  __device__ __forceinline__ void flush(char* out, long ld_bytes, long row0, long col_bytes, long lim_bytes,
                                        bool fp32_add = false) const {
    __syncwarp();
    const long cb = col_bytes + (lane & 7) * 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const long r = row0 + lane / 8 + 4 * i;
      if (r < out_rows && cb < lim_bytes) {
        uint4* dst = reinterpret_cast<uint4*>(out + r * ld_bytes + cb);
        uint4 val = *moved(i);
        if (fp32_add) {
          const uint4 old = *dst;
          val = make_uint4(__float_as_uint(__uint_as_float(val.x) + __uint_as_float(old.x)),
                           __float_as_uint(__uint_as_float(val.y) + __uint_as_float(old.y)),
                           __float_as_uint(__uint_as_float(val.z) + __uint_as_float(old.z)),
                           __float_as_uint(__uint_as_float(val.w) + __uint_as_float(old.w)));
        }
        *dst = val;
      }
    }
    __syncwarp();  // the box is free again
  }
  // 128 bytes of res rows row0 + r at col_bytes -> box, read back by the row owners with own()
  __device__ __forceinline__ void fetch(const char* res, long ld_bytes, long row0, long col_bytes) const {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const long r = row0 + lane / 8 + 4 * i;
      *moved(i) = r < out_rows ? *reinterpret_cast<const uint4*>(res + r * ld_bytes + col_bytes + (lane & 7) * 16)
                               : make_uint4(0, 0, 0, 0);
    }
    __syncwarp();
  }
};

// Optional per-tile timestamps of CTA 0 (clock64 of its SM) for tuning: null unless armed from the host
// (gemm_trace). Slots per tile: 0/1 producer first wait / last load issued, 2/3 issuer before / after the
// accumulator-free wait, 4 first k-block landed, 5 last MMA committed, 6/7 epilogue start / end.
constexpr int kTraceTiles = 64;
static __device__ unsigned long long* g_gemm_trace;

__device__ __forceinline__ void trace_mark(unsigned long long* tr, int local_tile, int slot) {
  if (tr && local_tile < kTraceTiles) tr[local_tile * 8 + slot] = clock64();
}

struct TileInfo {
  int group;
  int m_tile;
  int n_tile;
  int rows;      // valid rows of this tile (kGroupM) or K extent (kGroupK)
  int row0;      // first A row (kGroupM) / first K row (kGroupK)
  int num_kb;
};

template <int BN, int MODE>
__device__ __forceinline__ bool tile_info(const Params& p, const int* s_prefix, int ngroups, int tile, TileInfo& t) {
  if (MODE == kGroupM) {
    if (tile >= s_prefix[ngroups]) return false;
    int lo = 0, hi = ngroups - 1;
    while (lo < hi) {  // last g with prefix[g] <= tile
      int mid = (lo + hi + 1) >> 1;
      if (s_prefix[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int local = tile - s_prefix[g];
    t.group = g;
    t.m_tile = local / p.n_tiles;
    t.n_tile = local % p.n_tiles;
    const int grows = p.group_rows ? p.group_rows[g] : p.M;
    const int goff = p.group_off ? p.group_off[g] : 0;
    t.row0 = goff + t.m_tile * kBM;
    t.rows = min(kBM, grows - t.m_tile * kBM);
    t.num_kb = (p.K + kBK - 1) / kBK;
  } else {
    const int per_group = p.m_tiles * p.n_tiles;
    if (tile >= per_group * ngroups) return false;
    const int g = tile / per_group;
    const int local = tile % per_group;
    t.group = g;
    t.m_tile = local / p.n_tiles;
    t.n_tile = local % p.n_tiles;
    if (p.k_segments > 1) {
      int kb = 0;
      for (int sgi = 0; sgi < p.k_segments; ++sgi) kb += (p.group_rows[sgi * ngroups + g] + kBK - 1) / kBK;
      t.row0 = 0;
      t.rows = 0;
      t.num_kb = kb;
    } else if (!p.group_rows && p.k_chunk > 0) {
      t.row0 = g * p.k_chunk;
      t.rows = min(p.k_chunk, p.K - t.row0);
      t.num_kb = (t.rows + kBK - 1) / kBK;
    } else {
      const int krows = p.group_rows ? p.group_rows[g] : p.K;
      t.row0 = p.group_off ? p.group_off[g] : 0;
      t.rows = krows;
      t.num_kb = (krows + kBK - 1) / kBK;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------------------------------------
// epilogues: one thread = one accumulator row
// ---------------------------------------------------------------------------------------------------------
// TMA variant of the store and SwiGLU epilogues (bf16 out, no read-modify-write accumulation, local memory)
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile_tma(const Params& p, const TileInfo& t, uint32_t tmem_acc,
                                                  int row_in_tile, int warp_lane_base, TmaEpi& e, int lane) {
  const bool row_ok = row_in_tile < t.rows;
  const uint32_t tbase = tmem_acc + (static_cast<uint32_t>(warp_lane_base) << 16);
  if (EPI == kEpiStore) {
    const bool empty_k = (t.num_kb == 0);
    const int n0 = t.n_tile * BN;
#pragma unroll 1
    for (int c = 0; c < BN; c += 64) {
      float v[64];
      if (!empty_k) {
        tmem_ld32_pair(tbase + c, tbase + c + 32, v, v + 32);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = 0.f;
      }
      if (n0 + c >= p.N) continue;  // warp-uniform: the whole box lies past the last column
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        float x = row_ok ? v[i] * p.alpha : 0.f;
        if (row_ok && p.bias) x += (n0 + c + i < p.N) ? p.bias[n0 + c + i] : 0.f;
        v[i] = x;
      }
      box_acquire(lane);
      if (p.residual) {  // the residual box comes in through the same shared memory
        if (lane == 0) {
          mbar_arrive_expect_tx(e.res_bar, kStgBytes);
          tma_load_2d(e.box.base, e.map_res, e.res_bar, n0 + c, e.row);
        }
        const bool landed = mbar_wait(e.res_bar, e.res_phase, kTimeoutFull);
        e.res_phase ^= 1;
        if (landed && row_ok) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 r = *e.box.chunk(q);
            const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[8 * q + i] += __bfloat162float(rb[i]);
          }
        }
        __syncwarp();
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *e.box.chunk(q) = make_uint4(pack_bf16(v[8 * q], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                                     pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7]));
      box_release(e, e.map_out, n0 + c, lane);
    }
  } else {  // kEpiSwiGLU: acc columns [0, BN/2) = gate, [BN/2, BN) = up for FFN columns f0 + [0, BN/2)
    constexpr int HALF = BN / 2;
    const int f0 = t.n_tile * HALF;
#pragma unroll 1
    for (int c = 0; c < HALF; c += 64) {
      float g[64], u[64];
      tmem_ld32_pair(tbase + c, tbase + c + 32, g, g + 32);
      tmem_ld32_pair(tbase + HALF + c, tbase + HALF + c + 32, u, u + 32);
      if (f0 + c >= p.ffn) continue;
      if (!row_ok) {
#pragma unroll
        for (int i = 0; i < 64; ++i) { g[i] = 0.f; u[i] = 0.f; }
      }
      box_acquire(lane);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float hv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float gv = g[8 * q + i];
          hv[i] = __fdividef(gv, 1.0f + __expf(-gv)) * u[8 * q + i];
        }
        *e.box.chunk(q) = make_uint4(pack_bf16(hv[0], hv[1]), pack_bf16(hv[2], hv[3]), pack_bf16(hv[4], hv[5]),
                                     pack_bf16(hv[6], hv[7]));
      }
      box_release(e, e.map_out, f0 + c, lane);
      if (p.gu_out) {  // raw gate and up halves, two more boxes through the same staging
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          const float* src = half ? u : g;
          box_acquire(lane);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *e.box.chunk(q) = make_uint4(pack_bf16(src[8 * q], src[8 * q + 1]), pack_bf16(src[8 * q + 2], src[8 * q + 3]),
                                         pack_bf16(src[8 * q + 4], src[8 * q + 5]),
                                         pack_bf16(src[8 * q + 6], src[8 * q + 7]));
          box_release(e, e.map_gu, half * p.ffn + f0 + c, lane);
        }
      }
    }
  }
}

// Staged variant of the store and SwiGLU epilogues (N a multiple of 8; bf16 out without read-modify-write, or fp32
// out with or without it; local memory). kGroupK writes group g's block at out + g * out_group_stride.
template <int BN, int MODE, int EPI>
__device__ __forceinline__ void epilogue_tile_staged(const Params& p, const TileInfo& t, uint32_t tmem_acc,
                                                     int row_in_tile, int warp_lane_base, const StagedEpi& e) {
  const uint32_t tbase = tmem_acc + (static_cast<uint32_t>(warp_lane_base) << 16);
  if (EPI == kEpiStore) {
    const bool empty_k = (t.num_kb == 0);
    const int n0 = t.n_tile * BN;
    const long row0 = (MODE == kGroupM ? t.row0 : static_cast<long>(t.m_tile) * kBM) + warp_lane_base;
    const bool row_ok = MODE == kGroupM ? row_in_tile < t.rows : row0 + (row_in_tile - warp_lane_base) < p.M;
    const int esize = p.out_fp32 ? 4 : 2;
    char* out = static_cast<char*>(p.out);
    if (MODE == kGroupK) out += static_cast<long>(t.group) * p.out_group_stride * esize;
    const long ld_bytes = p.ldo * esize, lim_bytes = static_cast<long>(p.N) * esize;
#pragma unroll 1
    for (int c = 0; c < BN; c += 64) {
      float v[64];
      if (!empty_k) {
        tmem_ld32_pair(tbase + c, tbase + c + 32, v, v + 32);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = 0.f;
      }
      const int col = n0 + c;
      if (col >= p.N) continue;  // warp-uniform: the box lies past the last column
      const bool full = col + 64 <= p.N;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        float x = row_ok ? v[i] * p.alpha : 0.f;
        if (row_ok && p.bias) x += (full || col + i < p.N) ? p.bias[col + i] : 0.f;
        v[i] = x;
      }
      if (p.out_fp32) {  // two boxes of 32 fp32 columns
        e.put_f32(v);
        e.flush(out, ld_bytes, row0, static_cast<long>(col) * 4, lim_bytes, p.accumulate != 0);
        if (col + 32 < p.N) {
          e.put_f32(v + 32);
          e.flush(out, ld_bytes, row0, static_cast<long>(col + 32) * 4, lim_bytes, p.accumulate != 0);
        }
        continue;
      }
      if (p.residual) {  // the residual box comes in through the same shared memory, coalesced
        e.fetch(reinterpret_cast<const char*>(p.residual), p.ldr * 2, row0, static_cast<long>(col) * 2);
        if (row_ok) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 r = *e.own(q);
            const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[8 * q + i] += __bfloat162float(rb[i]);
          }
        }
        __syncwarp();
      }
      e.put(v);
      e.flush(out, ld_bytes, row0, static_cast<long>(col) * 2, lim_bytes);
    }
  } else {  // kEpiSwiGLU: acc columns [0, BN/2) = gate, [BN/2, BN) = up for FFN columns f0 + [0, BN/2)
    constexpr int HALF = BN / 2;
    const int f0 = t.n_tile * HALF;
    const bool row_ok = row_in_tile < t.rows;
    const long row0 = t.row0 + warp_lane_base;
    char* h = static_cast<char*>(p.out);
#pragma unroll 1
    for (int c = 0; c < HALF; c += 64) {
      if (f0 + c >= p.ffn) break;  // warp-uniform (F is a multiple of 64 on this path)
      float g[64], u[64];
      tmem_ld32_pair(tbase + c, tbase + c + 32, g, g + 32);
      tmem_ld32_pair(tbase + HALF + c, tbase + HALF + c + 32, u, u + 32);
      if (!row_ok) {
#pragma unroll
        for (int i = 0; i < 64; ++i) { g[i] = 0.f; u[i] = 0.f; }
      }
      if (p.gu_out) {  // raw gate and up rows first (g and u are overwritten below)
        char* gu = reinterpret_cast<char*>(p.gu_out);
        e.put(g);
        e.flush(gu, 4L * p.ffn, row0, 2L * (f0 + c), 4L * p.ffn);
        e.put(u);
        e.flush(gu, 4L * p.ffn, row0, 2L * (p.ffn + f0 + c), 4L * p.ffn);
      }
#pragma unroll
      for (int i = 0; i < 64; ++i) g[i] = __fdividef(g[i], 1.0f + __expf(-g[i])) * u[i];
      e.put(g);
      e.flush(h, p.ldo * 2, row0, 2L * (f0 + c), 2L * p.ffn);
    }
  }
}

template <int BN, int MODE, int EPI>
__device__ __forceinline__ void epilogue_tile(const Params& p, const TileInfo& t, uint32_t tmem_acc, int row_in_tile,
                                              int warp_lane_base) {
  const bool empty_k = (t.num_kb == 0);
  if (EPI == kEpiStore) {
    long out_row;
    bool row_ok, row_write;
    if (MODE == kGroupM) {
      out_row = t.row0 + row_in_tile;
      row_ok = row_in_tile < t.rows;
      row_write = row_ok || p.zero_pad_rows;
    } else {
      out_row = static_cast<long>(t.m_tile) * kBM + row_in_tile;
      row_ok = out_row < p.M;
      row_write = row_ok;
    }
    const int n0 = t.n_tile * BN;
    char* base = static_cast<char*>(p.out);
    if (MODE == kGroupK) base += static_cast<long>(t.group) * p.out_group_stride * (p.out_fp32 ? 4 : 2);
    long dst_row = out_row;
    if (MODE == kGroupM && p.peer_out && row_write) {
      const long owner = out_row / p.peer_rows;
      base = static_cast<char*>(p.peer_out[owner]);
      dst_row = static_cast<long>(p.peer_slot) * p.peer_rows + (out_row - owner * p.peer_rows);
    }
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      if (!empty_k) {
        tmem_ld32(tmem_acc + (static_cast<uint32_t>(warp_lane_base) << 16) + c, v);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      if (!row_write || n0 + c >= p.N) continue;
      const bool full = (n0 + c + 32 <= p.N);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float x = row_ok ? v[i] * p.alpha : 0.f;
        if (row_ok && p.bias && (full || n0 + c + i < p.N)) x += p.bias[n0 + c + i];
        v[i] = x;
      }
      if (row_ok && p.residual) {
        const __nv_bfloat16* r = p.residual + out_row * p.ldr + n0 + c;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (full || n0 + c + i < p.N) v[i] += __bfloat162float(r[i]);
      }
      if (p.out_fp32) {
        float* o = reinterpret_cast<float*>(base) + dst_row * p.ldo + n0 + c;
        if (full && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 w = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            if (p.accumulate) {
              float4 old = *reinterpret_cast<float4*>(o + i);
              w.x += old.x; w.y += old.y; w.z += old.z; w.w += old.w;
            }
            *reinterpret_cast<float4*>(o + i) = w;
          }
        } else {
          for (int i = 0; i < 32; ++i)
            if (n0 + c + i < p.N) o[i] = p.accumulate ? o[i] + v[i] : v[i];
        }
      } else {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(base) + dst_row * p.ldo + n0 + c;
        if (full && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            if (p.accumulate) {
              uint4 old = *reinterpret_cast<uint4*>(o + i);
              const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&old);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i + j] += __bfloat162float(ob[j]);
            }
            uint4 w;
            w.x = pack_bf16(v[i], v[i + 1]);
            w.y = pack_bf16(v[i + 2], v[i + 3]);
            w.z = pack_bf16(v[i + 4], v[i + 5]);
            w.w = pack_bf16(v[i + 6], v[i + 7]);
            *reinterpret_cast<uint4*>(o + i) = w;
          }
        } else {
          for (int i = 0; i < 32; ++i)
            if (n0 + c + i < p.N) {
              float x = v[i];
              if (p.accumulate) x += __bfloat162float(o[i]);
              o[i] = __float2bfloat16(x);
            }
        }
      }
    }
  } else if (EPI == kEpiSwiGLU) {
    // acc columns [0, BN/2) = gate, [BN/2, BN) = up for FFN columns f0 + [0, BN/2)
    constexpr int HALF = BN / 2;
    const long out_row = t.row0 + row_in_tile;
    const bool row_ok = row_in_tile < t.rows;
    const bool row_write = row_ok || p.zero_pad_rows;
    const int f0 = t.n_tile * HALF;
#pragma unroll 1
    for (int c = 0; c < HALF; c += 32) {
      float g[32], u[32];
      tmem_ld32(tmem_acc + (static_cast<uint32_t>(warp_lane_base) << 16) + c, g);
      tmem_ld32(tmem_acc + (static_cast<uint32_t>(warp_lane_base) << 16) + HALF + c, u);
      if (!row_write || f0 + c >= p.ffn) continue;
      const bool full = (f0 + c + 32 <= p.ffn);
      __nv_bfloat16* h = static_cast<__nv_bfloat16*>(p.out) + out_row * p.ldo + f0 + c;
      __nv_bfloat16* gu = p.gu_out ? p.gu_out + out_row * (2L * p.ffn) + f0 + c : nullptr;
      if (full) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w, wg, wu;
          float hv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) hv[j] = row_ok ? silu(g[i + j]) * u[i + j] : 0.f;
          w.x = pack_bf16(hv[0], hv[1]); w.y = pack_bf16(hv[2], hv[3]);
          w.z = pack_bf16(hv[4], hv[5]); w.w = pack_bf16(hv[6], hv[7]);
          *reinterpret_cast<uint4*>(h + i) = w;
          if (gu) {
            const float zg = row_ok ? 1.f : 0.f;
            wg.x = pack_bf16(zg * g[i], zg * g[i + 1]); wg.y = pack_bf16(zg * g[i + 2], zg * g[i + 3]);
            wg.z = pack_bf16(zg * g[i + 4], zg * g[i + 5]); wg.w = pack_bf16(zg * g[i + 6], zg * g[i + 7]);
            wu.x = pack_bf16(zg * u[i], zg * u[i + 1]); wu.y = pack_bf16(zg * u[i + 2], zg * u[i + 3]);
            wu.z = pack_bf16(zg * u[i + 4], zg * u[i + 5]); wu.w = pack_bf16(zg * u[i + 6], zg * u[i + 7]);
            *reinterpret_cast<uint4*>(gu + i) = wg;
            *reinterpret_cast<uint4*>(gu + p.ffn + i) = wu;
          }
        }
      } else {
        for (int i = 0; i < 32; ++i) {
          if (f0 + c + i >= p.ffn) break;
          h[i] = __float2bfloat16(row_ok ? silu(g[i]) * u[i] : 0.f);
          if (gu) {
            gu[i] = __float2bfloat16(row_ok ? g[i] : 0.f);
            gu[p.ffn + i] = __float2bfloat16(row_ok ? u[i] : 0.f);
          }
        }
      }
    }
  } else {  // kEpiSwiGLUBwd
    const long row = t.row0 + row_in_tile;
    const bool row_ok = row_in_tile < t.rows;
    const bool row_write = row_ok || p.zero_pad_rows;
    const int f0 = t.n_tile * BN;
    const float w = row_ok ? p.route_w[row] : 0.f;
    float dot = 0.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float a[32];
      tmem_ld32(tmem_acc + (static_cast<uint32_t>(warp_lane_base) << 16) + c, a);
      if (!row_write || f0 + c >= p.ffn) continue;
      const int lim = min(32, p.ffn - (f0 + c));
      const __nv_bfloat16* gp = p.gu_in + row * (2L * p.ffn) + f0 + c;
      __nv_bfloat16* dg = static_cast<__nv_bfloat16*>(p.out) + row * (2L * p.ffn) + f0 + c;
      __nv_bfloat16* hp = p.h_out ? p.h_out + row * static_cast<long>(p.ffn) + f0 + c : nullptr;
      for (int i0 = 0; i0 < lim; i0 += 8) {
        float gv[8], uv[8];
        if (i0 + 8 <= lim) {
          uint4 graw = *reinterpret_cast<const uint4*>(gp + i0);
          uint4 uraw = *reinterpret_cast<const uint4*>(gp + p.ffn + i0);
          const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&graw);
          const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uraw);
#pragma unroll
          for (int j = 0; j < 8; ++j) { gv[j] = __bfloat162float(gb[j]); uv[j] = __bfloat162float(ub[j]); }
        } else {
          for (int j = 0; j < 8; ++j) {
            gv[j] = (i0 + j < lim) ? __bfloat162float(gp[i0 + j]) : 0.f;
            uv[j] = (i0 + j < lim) ? __bfloat162float(gp[p.ffn + i0 + j]) : 0.f;
          }
        }
        float dgv[8], duv[8], hv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float sg = 1.f / (1.f + __expf(-gv[j]));
          const float sl = gv[j] * sg;
          hv[j] = sl * uv[j];
          const float dh = row_ok ? w * a[i0 + j] : 0.f;
          dot += row_ok ? a[i0 + j] * hv[j] : 0.f;
          duv[j] = dh * sl;
          dgv[j] = dh * uv[j] * (sg + sl * (1.f - sg));
          hv[j] = row_ok ? w * hv[j] : 0.f;  // router-weighted H feeds the down-projection weight gradient
        }
        if (i0 + 8 <= lim) {
          uint4 o1, o2;
          o1.x = pack_bf16(dgv[0], dgv[1]); o1.y = pack_bf16(dgv[2], dgv[3]);
          o1.z = pack_bf16(dgv[4], dgv[5]); o1.w = pack_bf16(dgv[6], dgv[7]);
          o2.x = pack_bf16(duv[0], duv[1]); o2.y = pack_bf16(duv[2], duv[3]);
          o2.z = pack_bf16(duv[4], duv[5]); o2.w = pack_bf16(duv[6], duv[7]);
          *reinterpret_cast<uint4*>(dg + i0) = o1;
          *reinterpret_cast<uint4*>(dg + p.ffn + i0) = o2;
          if (hp) {
            uint4 o3;
            o3.x = pack_bf16(hv[0], hv[1]); o3.y = pack_bf16(hv[2], hv[3]);
            o3.z = pack_bf16(hv[4], hv[5]); o3.w = pack_bf16(hv[6], hv[7]);
            *reinterpret_cast<uint4*>(hp + i0) = o3;
          }
        } else {
          for (int j = 0; j < 8 && i0 + j < lim; ++j) {
            dg[i0 + j] = __float2bfloat16(dgv[j]);
            dg[p.ffn + i0 + j] = __float2bfloat16(duv[j]);
            if (hp) hp[i0 + j] = __float2bfloat16(hv[j]);
          }
        }
      }
    }
    if (p.dw_partial && row_write) p.dw_partial[row * p.n_tiles + t.n_tile] = dot;
  }
}

// ---------------------------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------------------------
template <int BN, int MODE, int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_out, const __grid_constant__ CUtensorMap map_res,
                const __grid_constant__ CUtensorMap map_gu, Params p) {
  using S = Smem<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* teardown = acc_empty + 2;
  uint64_t* res_full = teardown + 1;  // [4] residual boxes of the epilogue warps (TMA epilogue)
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(res_full + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  __shared__ int s_prefix[1025];

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int ngroups = p.num_groups;
  unsigned long long* const trace = blockIdx.x == 0 ? g_gemm_trace : nullptr;

  // group prefix (tiles before each group) for kGroupM
  if (MODE == kGroupM && threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < ngroups; ++g) {
      s_prefix[g] = acc;
      const int rows = p.group_rows ? p.group_rows[g] : p.M;
      acc += ((rows + kBM - 1) / kBM) * p.n_tiles;
    }
    s_prefix[ngroups] = min(acc, p.max_tiles);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(teardown, 1);
    for (int w = 0; w < 4; ++w) mbar_init(&res_full[w], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    if (p.tma_out) {
      tma_prefetch_desc(&map_out);
      if (p.residual) tma_prefetch_desc(&map_res);
      if (p.gu_out) tma_prefetch_desc(&map_gu);
    }
  }
  if (warp == 1) tmem_alloc(tmem_base_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued_phase[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) issued_phase[s] = -1;
      TileInfo t;
      int local = 0;
      for (int tile = blockIdx.x; !*abort_flag && tile_info<BN, MODE>(p, s_prefix, ngroups, tile, t);
           tile += gridDim.x, ++local) {
        trace_mark(trace, local, 0);
        for (int kb = 0; kb < t.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, kTimeoutEmpty)) { *abort_flag = 1; break; }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          issued_phase[stage] = static_cast<int>(phase);
          if (MODE == kGroupM) {
            const int k0 = kb * kBK;
            if (!A_MN) {
              tma_load_2d(sa, &map_a, &full[stage], k0, t.row0);
            } else {
              tma_load_2d(sa, &map_a, &full[stage], t.row0, k0);
              tma_load_2d(sa + S::kABytes / 2, &map_a, &full[stage], t.row0 + 64, k0);
            }
            const int bgroup = p.expert_mod > 0 ? t.group % p.expert_mod : t.group;
            if (!B_MN) {
              const int brow = bgroup * p.b_group_rows;
              if (p.dual_b_offset > 0) {
                const int half = BN / 2;
                tma_load_2d(sb, &map_b, &full[stage], k0, brow + t.n_tile * half);
                tma_load_2d(sb + S::kBBytes / 2, &map_b, &full[stage], k0, brow + p.dual_b_offset + t.n_tile * half);
              } else {
                tma_load_2d(sb, &map_b, &full[stage], k0, brow + t.n_tile * BN);
              }
            } else {
              const int krow = bgroup * p.b_group_rows + k0;
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_2d(sb + j * (kBK * 64 * 2), &map_b, &full[stage], t.n_tile * BN + 64 * j, krow);
            }
          } else {  // kGroupK: both operands MN-major, K = rows
            int krow = t.row0 + kb * kBK;
            if (p.k_segments > 1) {  // walk the segments to find the one holding k-block kb
              int rem = kb;
              for (int sgi = 0; sgi < p.k_segments; ++sgi) {
                const int idx = sgi * ngroups + t.group;
                const int nkb = (p.group_rows[idx] + kBK - 1) / kBK;
                if (rem < nkb) { krow = p.group_off[idx] + rem * kBK; break; }
                rem -= nkb;
              }
            }
            tma_load_2d(sa, &map_a, &full[stage], t.m_tile * kBM, krow);
            tma_load_2d(sa + S::kABytes / 2, &map_a, &full[stage], t.m_tile * kBM + 64, krow);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * (kBK * 64 * 2), &map_b, &full[stage], t.n_tile * BN + 64 * j, krow);
          }
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        trace_mark(trace, local, 1);
      }
      // drain: every stage this thread filled must have landed before the CTA may exit
      for (int s = 0; s < kStages; ++s)
        if (issued_phase[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(issued_phase[s]), kTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      TileInfo t;
      int local = 0;
      for (int tile = blockIdx.x; !*abort_flag && tile_info<BN, MODE>(p, s_prefix, ngroups, tile, t);
           tile += gridDim.x, ++local) {
        trace_mark(trace, local, 2);
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, kTimeoutAccumFree)) { *abort_flag = 1; break; }
        trace_mark(trace, local, 3);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < t.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, kTimeoutFull)) { *abort_flag = 1; ok = false; break; }
          if (kb == 0) trace_mark(trace, local, 4);
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            uint64_t da, db;
            if (!A_MN) da = smem_desc_sw128(sa + k * 32, 16, 1024);
            else       da = smem_desc_sw128(sa + k * 2048, 8192, 1024);
            if (!B_MN) db = smem_desc_sw128(sb + k * 32, 16, 1024);
            else       db = smem_desc_sw128(sb + k * 2048, 8192, 1024);
            umma_bf16(d_tmem, da, db, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        umma_commit(&acc_full[acc]);
        trace_mark(trace, local, 5);
        if (!ok) break;
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      // all issued MMAs must finish before TMEM is released
      umma_commit(teardown);
      mbar_wait(teardown, 0, kTimeoutAccum);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int lane_base = 32 * (warp % 4);
    const int row_in_tile = lane_base + lane;
    const StagedEpi se{smem + S::kStg + (warp % 4) * kStgBytes, lane,
                       (MODE == kGroupM && p.group_rows) ? LONG_MAX : static_cast<long>(p.M)};
    TmaEpi te{{smem + S::kStg + (warp % 4) * kStgBytes, lane}, &map_out, &map_res, &map_gu, &res_full[warp % 4], 0u, 0};
    int acc = 0;
    uint32_t acc_phase = 0;
    TileInfo t;
    unsigned long long* const etrace = threadIdx.x == 64 ? trace : nullptr;
    int local = 0;
    for (int tile = blockIdx.x; tile_info<BN, MODE>(p, s_prefix, ngroups, tile, t); tile += gridDim.x, ++local) {
      if (*abort_flag) break;
      if (!mbar_wait(&acc_full[acc], acc_phase, kTimeoutAccum)) { *abort_flag = 1; break; }
      trace_mark(etrace, local, 6);
      tc_fence_after();
      if constexpr (MODE == kGroupM && EPI != kEpiSwiGLUBwd) {
        if (p.tma_out) {
          te.row = t.row0 + lane_base;
          epilogue_tile_tma<BN, EPI>(p, t, tmem_base + acc * BN, row_in_tile, lane_base, te, lane);
          trace_mark(etrace, local, 7);
          tc_fence_before();
          mbar_arrive(&acc_empty[acc]);
          if (++acc == 2) { acc = 0; acc_phase ^= 1; }
          continue;
        }
      }
      if constexpr (EPI == kEpiStore || (MODE == kGroupM && EPI == kEpiSwiGLU)) {
        if (p.staged_out) {
          epilogue_tile_staged<BN, MODE, EPI>(p, t, tmem_base + acc * BN, row_in_tile, lane_base, se);
        } else {
          epilogue_tile<BN, MODE, EPI>(p, t, tmem_base + acc * BN, row_in_tile, lane_base);
        }
      } else {
        epilogue_tile<BN, MODE, EPI>(p, t, tmem_base + acc * BN, row_in_tile, lane_base);
      }
      trace_mark(etrace, local, 7);
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    // rows stored into peers' memory are made visible at system scope before the kernel ends, so the flag that a
    // later kernel releases to the peers orders them
    if (p.peer_out) __threadfence_system();
    if (p.tma_out && lane == 0) tma_store_wait_all();  // bulk stores complete before the CTA (and its smem) is gone
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 2 * BN);
}

}  // namespace gemm
}  // namespace qw
