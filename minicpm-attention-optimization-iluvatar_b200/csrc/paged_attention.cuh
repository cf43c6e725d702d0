// paged_attention.cuh -- causal varlen paged prefill attention for sm_100a.
//
// Semantics follow the reference Split-KV kernel
// (kernels/triton_split_kv_paged.py:63-155 of the reference project):
//   * query row i of sequence b sits at absolute position L_b - q_len_b + i;
//   * a key is valid for a row iff it is inside the row's split and <= the
//     row's absolute position; a row with no valid key keeps l = 0 and O = 0;
//   * an unsplit unit writes the normalised output directly; a unit split
//     s ways writes, per split, the normalised partial O (in the query
//     dtype) plus m (natural-log units) and l, which unit_combine_kernel
//     reduces with the weights of the reference's _split_kv_reduce.
// Splits are chosen per query unit by the schedule kernel: the caller's
// num_splits is the most any unit gets, and a unit is split only when it is a
// large share of the batch's work per SM (so a batch that fills the GPU many
// times over runs unsplit).  A unit split s ways covers its own key range
// [0, min(L, last row's position + 1)) in s runs of whole 128-key tiles (the
// reference splits [0, L) into ceil(L/S)-key runs; the combined output is the
// same attention, within rounding).
//
// Work unit = (sequence, KV head, query-tile pair, split).  A query tile packs
// the G = Hq / KH query heads that share one KV head with P = floor(128 / G)
// query positions into the rows of one 128-row UMMA M dimension (row r =
// position r / G, head r % G; rows past G x P are zero padding when G does not
// divide 128), so every K/V tile fetched feeds all G heads.  A unit
// holds two such tiles (2P consecutive positions, 256 rows) that share every
// K/V tile; the second is skipped when the sequence has no rows for it.
//
// Persistent CTAs, one per SM, each looping over units that it claims from
// the heaviest-first work list (attn_schedule_kernel) with an atomic counter;
// 12 warps in 3 warpgroups:
//   warp 0      producer: claims a unit and publishes it in a 4-entry
//               shared-memory ring, then issues the TMA copies: Q0/Q1 once
//               the previous unit's last S is issued (Q_EMPTY), then K_j and
//               V_j tiles of 128 tokens into a 5-slot ring, each tile as 8
//               page slices of 16 tokens x 2 half-rows (a per-page gather
//               through the block table).  Slices past the unit's last key
//               use an out-of-range page index, so TMA fills zeros and reads
//               nothing outside the cache.  The next unit's copies therefore
//               overlap the current unit's last tiles and epilogue.
//   warp 1      TMEM owner and single-thread UMMA issuer, in the order
//               S0(j+1) = Q0 K^T after PV0(j), S1(j+1) after PV1(j), so each
//               softmax warpgroup works while the tensor core runs the other
//               tile's MMAs.  O_t += P_t V with P read from TMEM (TS form).
//   warps 2..3  idle (they complete the first warpgroup for setmaxnreg)
//   warps 4..7  softmax warpgroup of tile 0, warps 8..11 of tile 1; one query
//               row per thread: S row from TMEM, mask, online softmax in base
//               2, P (bf16/f16) written back over the S columns in TMEM.  The
//               running maximum is raised only when a row maximum grows by
//               more than 2^8; only then is O rescaled (rare after the first
//               tile).  Final normalise and store.
// Barrier phases run on counters kept across units: K/V ring fills, Q loads,
// and tiles per query tile (S_FULL, P_FULL, O_DONE).  A unit's first PV
// overwrites O_t only after tile t's softmax warps have published its first
// P, which they do after their epilogue has read the previous unit's O_t.
// TMEM: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512); P_t in the
// first 64 columns of S_t.
// Registers: launched at 168 per thread (the 384-thread limit); the first
// warpgroup gives back down to 104 and the softmax warpgroups take 200 each
// (104 + 2 x 200 = 3 x 168, the launch's total).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "sm100_ptx.cuh"
#include "split_combine.cuh"

namespace b200 {

constexpr int kAttnTileM = 128;   // rows per query tile
constexpr int kAttnTileN = 128;   // KV tokens per tile
constexpr int kAttnHeadDim = 128; // head_dim handled by this kernel
constexpr int kAttnSlice = 16;    // KV tokens per TMA box (page slice)
constexpr int kAttnTilesPerUnit = 2;
constexpr int kAttnThreads = 384;
constexpr int kAttnLaunchRegs = 168;   // 65536 / 384 rounded down to a multiple of 8
constexpr int kAttnProducerRegs = 104;
constexpr int kAttnSoftmaxRegs = 200;
static_assert(kAttnProducerRegs + 2 * kAttnSoftmaxRegs == 3 * kAttnLaunchRegs, "register split");
constexpr int kAttnTmemCols = 512;
constexpr int kKvStages = 5;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8
constexpr float kRescaleSum = 256.0f;      // 2^kRescaleThreshold

// Shared memory map (offsets from a 1024-aligned base).
constexpr uint32_t kSmQ = 0;                            // Q0, Q1: 2 x (2 x 16 KB)
constexpr uint32_t kSmKV = 65536;                       // ring: kKvStages x 32 KB
constexpr uint32_t kSmBar = kSmKV + kKvStages * 32768;  // mbarriers, TMEM slot, abort flag, unit ring
constexpr uint32_t kSmBytes = kSmBar + 512;
constexpr uint32_t kAttnSmemAlloc = kSmBytes + 1024;    // + alignment slack
static_assert(kAttnSmemAlloc <= 232448, "shared memory per CTA");
constexpr int kUnitRing = 4;  // claimed work units in flight between the producer and the consumers

enum : int {
  BAR_Q_FULL = 0,
  BAR_Q_EMPTY = 1,
  BAR_KV_FULL = 2,                           // + slot
  BAR_KV_EMPTY = BAR_KV_FULL + kKvStages,    // + slot
  BAR_S_FULL = BAR_KV_EMPTY + kKvStages,     // + tile
  BAR_P_FULL = BAR_S_FULL + 2,               // + 2 * tile + half (64 keys of P)
  BAR_O_DONE = BAR_P_FULL + 4,               // + tile
  BAR_IT_FULL = BAR_O_DONE + 2,              // + ring entry
  BAR_IT_EMPTY = BAR_IT_FULL + kUnitRing,    // + ring entry
  BAR_DRAIN = BAR_IT_EMPTY + kUnitRing,
  BAR_COUNT = BAR_DRAIN + 1
};

// A claimed unit as the producer publishes it: (seq, qunit, kvh, split, the
// unit's split count, its partial-output slot), then cu_q[seq], cu_q[seq + 1],
// seqused[seq] and a valid flag (0 ends the loop).
struct UnitEntry {
  int seq, qunit, kvh, split, nsplit, slot, q_begin, q_end, seq_len, valid;
};

// Work-list entry: x = sequence, y = query unit, z = KV head | split << 16 |
// split count << 24, w = partial-output slot of a split unit (-1 unsplit).
__device__ __forceinline__ int4 pack_unit(int seq, int qunit, int kvh, int split, int nsplit, int slot) {
  return make_int4(seq, qunit, kvh | (split << 16) | (nsplit << 24), slot);
}
__device__ __forceinline__ void unpack_unit(const int4 u, int& kvh, int& split, int& nsplit) {
  kvh = u.z & 0xffff;
  split = (u.z >> 16) & 0xff;
  nsplit = (u.z >> 24) & 0xff;
}
constexpr int kUnitRows = 256;  // partial rows per split unit: 2 query tiles x 128 rows
constexpr uint32_t kSmRing = BAR_COUNT * 8 + 16;  // after the barriers, the TMEM slot and the abort flag
static_assert(kSmRing + kUnitRing * sizeof(UnitEntry) <= 512, "barrier area");

struct AttnKernelArgs {
  const void* block_table;
  const void* cu_q;
  const void* seqused;
  void* out;
  void* o_split;
  float* m_split;    // [slots][num_splits][kUnitRows]
  float* l_split;
  const int4* units;
  const int* unit_count;
  int64_t bt_stride;
  int64_t out_st, out_sh;
  int bt_cols;
  int bt_i64;
  int len_i64;
  int total_q;
  int num_q_heads;
  int group;          // G = Hq / KH, 1..128
  int pos_per_tile;   // P = floor(128 / G)
  int block_size;
  int num_blocks;
  int num_splits;     // the most splits any unit has (the partial buffers' split stride)
  int head_dim;       // 128, or 64 (the upper 64 columns of every tile are TMA zero fill)
  float scale_log2;   // softmax_scale * log2(e)
};

// K/V tensor maps.  Up to kMaxHeadMaps KV heads: one 5-D map per head,
// (d % 64, key % 8, half of head_dim, key / 8 in the page, page), whose box is
// a 16-key page slice with both halves (4 KB): 8 boxes per 128-key tile.  More
// heads: k[0] / v[0] hold a 4-D map (d, key in the page, head, page) whose box
// is one half of a slice (2 KB): 16 boxes per tile.  The TMA unit's per-box
// cost makes the box count matter (2 KB boxes instead of 4 KB cost 10 % at 16K).
constexpr int kMaxHeadMaps = 8;
struct KvHeadMaps {
  CUtensorMap k[kMaxHeadMaps];
  CUtensorMap v[kMaxHeadMaps];
};

// Shared-memory offset of the 16-byte piece `chunk` of row r (a key) of half h
// in one K/V ring slot.  Per-head maps: 8-key groups of 2 KB, each holding both
// halves (8 rows of 128 B each); 4-D maps: two 16 KB halves of 128 rows.
template <bool kHeadMaps, bool kNarrow = false>
__device__ __forceinline__ uint32_t kv_slot_offset(int r, int h, int chunk) {
  if (kNarrow) return r * 128 + chunk * 16;  // head_dim 64: one 64-column half, 128 B rows (both map kinds)
  return kHeadMaps ? (r >> 3) * 2048 + h * 1024 + (r & 7) * 128 + chunk * 16 : h * 16384 + r * 128 + chunk * 16;
}

__device__ __forceinline__ int load_index(const void* p, int64_t i, int is_i64) {
  return is_i64 ? static_cast<int>(static_cast<const int64_t*>(p)[i]) : static_cast<const int*>(p)[i];
}

// Geometry of one work unit (pos_per_unit consecutive query positions);
// shared by the scheduler (cost) and the kernel.
struct UnitGeom {
  int q_begin, q_len, seq_len;
  int pos0, split_begin, split_end;
  int kv_lo, kv_hi, n_tiles;
  int q_abs_min;
};

// KV tiles of a query unit's whole causal key range [0, min(L, last row + 1)).
__device__ __forceinline__ int qunit_full_tiles(int q_len, int seq_len, int qunit, int pos_per_unit) {
  const int pos0 = qunit * pos_per_unit;
  const int rows = min(pos_per_unit, q_len - pos0);
  const int kv_end = min(max(seq_len, 0), seq_len - q_len + pos0 + rows);
  return kv_end > 0 ? (kv_end + kAttnTileN - 1) / kAttnTileN : 0;
}

// Split `split` of `nsplit` covers whole tiles [split * tps, (split + 1) * tps)
// of the unit's key range, tps = ceil(full tiles / nsplit).
__device__ __forceinline__ UnitGeom unit_geometry(int q_begin, int q_end, int seq_len, int qunit, int split,
                                                  int nsplit, int pos_per_unit) {
  UnitGeom u;
  u.q_begin = q_begin;
  u.q_len = q_end - q_begin;
  u.seq_len = seq_len;
  u.pos0 = qunit * pos_per_unit;
  const int rows = min(pos_per_unit, u.q_len - u.pos0);
  u.q_abs_min = seq_len - u.q_len + u.pos0;
  const int kv_end = max(min(max(seq_len, 0), u.q_abs_min + rows), 0);
  const int n_full = (kv_end + kAttnTileN - 1) / kAttnTileN;
  const int tps = nsplit > 1 ? (n_full + nsplit - 1) / nsplit : n_full;
  u.split_begin = split * tps * kAttnTileN;
  u.split_end = min(u.split_begin + tps * kAttnTileN, kv_end);
  u.kv_hi = u.split_end;
  u.kv_lo = u.split_begin;
  u.n_tiles = (u.kv_hi > u.split_begin) ? (u.kv_hi - u.kv_lo + kAttnTileN - 1) / kAttnTileN : 0;
  return u;
}

template <typename T>
struct Pack2;
template <>
struct Pack2<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct Pack2<__half> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// Wait without the abort short-cut: used to let copies and MMAs already in
// flight land before the CTA exits.
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > B200_WAIT_LIMIT_NS) {
      record_device_error(B200_DEVERR_WAIT_TIMEOUT);
      return;
    }
  }
}

// kWide: head_dim 256.  A unit is then one query tile (TMEM: S 128 columns +
// O 256 columns, where the narrow kernel holds two S and two O), Q fills the
// whole 64 KB Q area (four 64-column quarters), and every KV tile takes four
// ring slots -- K and V each as two 128-column halves, each half in the narrow
// kernel's slot layout -- so S = Q K^T is 16 UMMAs over two K slots and
// O += P V two N = 128 UMMA chains, one per V half.  The second softmax
// warpgroup has no tile and idles.
//
// kNarrow: head_dim 64.  K/V tiles fill the first 16 KB of their ring slots (one
// 64-column half per row), S = Q K^T is 4 UMMAs (K = 64) and O += P V runs with
// N = 64 (O in the first 64 of the tile's 128 TMEM columns).
template <typename T, bool kHeadMaps, bool kWide, bool kNarrow>
__global__ void __launch_bounds__(kAttnThreads, 1)
    paged_attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ KvHeadMaps maps,
                          const AttnKernelArgs a) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kTilesPerUnit = kWide ? 1 : kAttnTilesPerUnit;
  constexpr int kFillsPerTile = kWide ? 4 : 2;  // ring slots per KV tile: K (, K hi), V (, V hi)
  griddep_wait();  // launched as a programmatic dependent of the schedule kernel

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmBar + BAR_COUNT * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmBar + BAR_COUNT * 8 + 4);
  volatile UnitEntry* ring = reinterpret_cast<volatile UnitEntry*>(smem + kSmBar + kSmRing);
  auto bar = [&](int i) { return smem_addr(&bars[i]); };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int P = a.pos_per_tile;
  const int ppu = kTilesPerUnit * P;

  if (threadIdx.x == 0) {
    mbar_init(bar(BAR_Q_FULL), 1);
    mbar_init(bar(BAR_Q_EMPTY), 1);
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(bar(BAR_KV_FULL + s), 1);
      mbar_init(bar(BAR_KV_EMPTY + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(BAR_S_FULL + t), 1);
      for (int h = 0; h < 2; ++h) mbar_init(bar(BAR_P_FULL + 2 * t + h), 4);
      mbar_init(bar(BAR_O_DONE + t), 1);
    }
    for (int r = 0; r < kUnitRing; ++r) {
      mbar_init(bar(BAR_IT_FULL + r), 1);
      mbar_init(bar(BAR_IT_EMPTY + r), 9);  // the MMA issuer and the 8 softmax warps
    }
    mbar_init(bar(BAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), kAttnTmemCols);
    tmem_relinquish();
  }
  // A query tile holds G x P (position, head) rows; with G not dividing 128
  // the last 128 - G x P rows are never loaded.  Zero them once so that their
  // (unstored) S rows stay finite and every softmax warp keeps its fast path.
  const int q_rows = a.group * P;
  if (q_rows < kAttnTileM) {
    const int pad = kAttnTileM - q_rows;
    for (int i = threadIdx.x; i < 4 * pad * 8; i += kAttnThreads) {  // 2 tiles x 2 halves x pad rows x 8 pieces
      const int r = q_rows + (i >> 3) % pad, part = (i >> 3) / pad;
      st_shared_v4(sbase + kSmQ + part * 16384 + r * 128 + (i & 7) * 16, 0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Consumers read ring entry it; false when the loop must end.
  auto take_entry = [&](int it, UnitEntry& e) -> bool {
    const int r = it % kUnitRing;
    if (!mbar_wait(bar(BAR_IT_FULL + r), (it / kUnitRing) & 1, abort_flag)) return false;
    e.seq = ring[r].seq;
    e.qunit = ring[r].qunit;
    e.kvh = ring[r].kvh;
    e.split = ring[r].split;
    e.nsplit = ring[r].nsplit;
    e.slot = ring[r].slot;
    e.q_begin = ring[r].q_begin;
    e.q_end = ring[r].q_end;
    e.seq_len = ring[r].seq_len;
    e.valid = ring[r].valid;
    return true;
  };
  auto geometry = [&](const UnitEntry& e) {
    return unit_geometry(e.q_begin, e.q_end, e.seq_len, e.qunit, e.split, e.nsplit, ppu);
  };

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAttnProducerRegs));
    if (warp == 0) {
      // ---------------------------------------------------------- producer (whole warp)
      if (lane == 0) tma_prefetch_desc(&tm_q);
      if (lane < (kHeadMaps ? a.num_q_heads / a.group : 1)) {
        tma_prefetch_desc(&maps.k[lane]);
        tma_prefetch_desc(&maps.v[lane]);
      }
      const int unit_count = *a.unit_count;
      int* claim = const_cast<int*>(a.unit_count) + 1;  // reset to 0 by the schedule kernel
      int issued = 0;   // K/V ring fills so far
      int q_loads = 0;  // Q loads so far
      const int my_slice = lane & 7;
      for (int it = 0;; ++it) {
        int u = 0;
        if (lane == 0) u = atomicAdd(claim, 1);
        u = __shfl_sync(0xffffffffu, u, 0);
        UnitEntry e{};
        e.valid = u < unit_count;
        if (e.valid) {
          const int4 un = a.units[u];
          e.seq = un.x;
          e.qunit = un.y;
          unpack_unit(un, e.kvh, e.split, e.nsplit);
          e.slot = un.w;
          e.q_begin = load_index(a.cu_q, e.seq, a.len_i64);
          e.q_end = load_index(a.cu_q, e.seq + 1, a.len_i64);
          e.seq_len = load_index(a.seqused, e.seq, a.len_i64);
        }
        int ok = 1;
        if (lane == 0) {
          const int r = it % kUnitRing;
          ok = mbar_wait(bar(BAR_IT_EMPTY + r), ((it / kUnitRing) & 1) ^ 1, abort_flag);
          if (ok) {
            ring[r].seq = e.seq;
            ring[r].qunit = e.qunit;
            ring[r].kvh = e.kvh;
            ring[r].split = e.split;
            ring[r].nsplit = e.nsplit;
            ring[r].slot = e.slot;
            ring[r].q_begin = e.q_begin;
            ring[r].q_end = e.q_end;
            ring[r].seq_len = e.seq_len;
            ring[r].valid = e.valid;
            mbar_arrive(bar(BAR_IT_FULL + r));  // release: the entry is visible to the waiters
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0) || !e.valid) break;
        const UnitGeom ug = geometry(e);
        const int n_tiles = ug.n_tiles;
        if (n_tiles == 0) continue;
        const bool two = !kWide && ug.pos0 + P < ug.q_len;
        if (lane == 0) {
          ok = mbar_wait(bar(BAR_Q_EMPTY), (q_loads & 1) ^ 1, abort_flag);
          if (ok) {
            const int head0 = e.kvh * a.group;
            const int t0 = ug.q_begin + ug.pos0;
            if (kWide) {  // one tile, four 64-column quarters of 128 B rows
              mbar_arrive_expect_tx(bar(BAR_Q_FULL), 4 * q_rows * 128);
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4)
                tma_load_3d(sbase + kSmQ + q4 * 16384, &tm_q, bar(BAR_Q_FULL), 64 * q4, head0, t0);
            } else if (kNarrow) {  // one 64-column box per tile
              mbar_arrive_expect_tx(bar(BAR_Q_FULL), (two ? 2 : 1) * q_rows * 128);
              tma_load_3d(sbase + kSmQ, &tm_q, bar(BAR_Q_FULL), 0, head0, t0);
              if (two) tma_load_3d(sbase + kSmQ + 32768, &tm_q, bar(BAR_Q_FULL), 0, head0, t0 + P);
            } else {
              mbar_arrive_expect_tx(bar(BAR_Q_FULL), (two ? 2 : 1) * q_rows * 256);  // 2 halves of 128 B rows
              tma_load_3d(sbase + kSmQ, &tm_q, bar(BAR_Q_FULL), 0, head0, t0);
              tma_load_3d(sbase + kSmQ + 16384, &tm_q, bar(BAR_Q_FULL), 64, head0, t0);
              if (two) {
                tma_load_3d(sbase + kSmQ + 32768, &tm_q, bar(BAR_Q_FULL), 0, head0, t0 + P);
                tma_load_3d(sbase + kSmQ + 49152, &tm_q, bar(BAR_Q_FULL), 64, head0, t0 + P);
              }
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        ++q_loads;
        const int64_t bt_row = static_cast<int64_t>(e.seq) * a.bt_stride;
        auto lookup = [&](int j, int& pg, int& of) {
          const int pos = ug.kv_lo + j * kAttnTileN + my_slice * kAttnSlice;
          const int lp = pos / a.block_size;
          of = pos - lp * a.block_size;
          const int lpc = min(lp, a.bt_cols - 1);
          const int v = load_index(a.block_table, bt_row + lpc, a.bt_i64);
          pg = (pos < ug.kv_hi && lp < a.bt_cols) ? v : a.num_blocks;
        };
        int pg_cur, of_cur, pg_nxt = a.num_blocks, of_nxt = 0;
        lookup(0, pg_cur, of_cur);
        if (n_tiles > 1) lookup(1, pg_nxt, of_nxt);
        bool stop = false;
        for (int idx = 0; idx < kFillsPerTile * n_tiles; ++idx) {
          const int j = idx / kFillsPerTile;
          const int part = idx % kFillsPerTile;  // K, V  or  K lo, K hi, V lo, V hi
          const bool is_v = part >= kFillsPerTile / 2;
          const int hi = kWide ? (part & 1) : 0;  // 128-column half of a head_dim-256 row
          const int slot = issued % kKvStages;
          const uint32_t ph = (issued / kKvStages) & 1;
          if (part == 0 && j > 0) {
            pg_cur = pg_nxt;
            of_cur = of_nxt;
            if (j + 1 < n_tiles) lookup(j + 1, pg_nxt, of_nxt);
          }
          // 4-D maps: lanes 0..15 issue half lane & 1 of slice (lane >> 1); head_dim 64: lane c < 8 slice c.
          const int c = kNarrow ? (lane & 7) : ((lane >> 1) & 7);
          const int page = kHeadMaps ? pg_cur : __shfl_sync(0xffffffffu, pg_cur, c);
          const int off = kHeadMaps ? of_cur : __shfl_sync(0xffffffffu, of_cur, c);
          if (lane == 0) {
            ok = mbar_wait(bar(BAR_KV_EMPTY + slot), ph ^ 1, abort_flag);
            if (ok) mbar_arrive_expect_tx(bar(BAR_KV_FULL + slot), kNarrow ? 16384 : 32768);
          }
          if (!__shfl_sync(0xffffffffu, ok, 0)) {  // also orders the expect_tx before the copies
            stop = true;
            break;
          }
          if (kHeadMaps) {
            // lane c < 8 issues slice c (its own lookup): 16 keys x both halves.
            if (lane < 8) {
              const CUtensorMap* map = is_v ? &maps.v[e.kvh] : &maps.k[e.kvh];
              tma_load_5d(sbase + kSmKV + slot * 32768 + lane * (kNarrow ? 2048 : 4096), map,
                          bar(BAR_KV_FULL + slot), 0, 0, 2 * hi, off >> 3, page);
            }
          } else if (lane < (kNarrow ? 8 : 16)) {
            const int half = kNarrow ? 0 : (lane & 1);
            const CUtensorMap* map = is_v ? &maps.v[0] : &maps.k[0];
            tma_load_4d(sbase + kSmKV + slot * 32768 + half * 16384 + c * 2048, map, bar(BAR_KV_FULL + slot),
                        half * 64 + hi * 128, off, e.kvh, page);
          }
          ++issued;
        }
        if (stop) break;
      }
      // Tail: every issued copy lands, and the UMMA commits that release the
      // slots arrive, before the CTA's shared memory is given back.
      if (lane == 0) {
        if (q_loads > 0) mbar_wait_drain(bar(BAR_Q_FULL), (q_loads - 1) & 1);
        for (int s = 0; s < kKvStages && s < issued; ++s) {
          const int last_idx = s + kKvStages * ((issued - 1 - s) / kKvStages);
          const uint32_t last = (last_idx / kKvStages) & 1;
          mbar_wait_drain(bar(BAR_KV_FULL + s), last);
          if (!*abort_flag) mbar_wait_drain(bar(BAR_KV_EMPTY + s), last);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_qk = umma_idesc_f16(kBF16, 128, 128, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_f16(kBF16, 128, kNarrow ? 64 : 128, false, true);
      constexpr int kQkSteps = kNarrow ? 4 : 8;  // K = 16 per UMMA over head_dim (64 or 128)
      constexpr uint32_t kKvSbo = kNarrow ? 1024 : (kHeadMaps ? 2048 : 1024);  // bytes between 8-key groups
      int fills = 0, q_uses = 0;
      int tiles_done[2] = {0, 0};  // tiles already processed by query-tile group t
      // Descriptors are built once per operand tile; the UMMAs of a tile step
      // their start address by adding (offset >> 4) to the descriptor's
      // address field (shared addresses stay below 256 KB, so the 14-bit field
      // never carries).  Every instruction between two UMMAs idles the tensor
      // core, which takes only about one UMMA ahead of execution.
      auto issue_s = [&](int t, uint32_t kslot_addr) {
        const uint64_t qd = umma_desc_sw128(sbase + kSmQ + t * 32768, 16, 1024);
        const uint64_t kd = umma_desc_sw128(kslot_addr, 16, kKvSbo);
#pragma unroll
        for (int kk = 0; kk < kQkSteps; ++kk) {
          const uint32_t qoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t koff = kv_slot_offset<kHeadMaps, kNarrow>(0, kk >> 2, 0) + (kk & 3) * 32;
          umma_ss(tmem + t * 128, qd + (qoff >> 4), kd + (koff >> 4), idesc_qk, kk > 0);
        }
        tc_commit(bar(BAR_S_FULL + t));
      };
      auto issue_pv = [&](int t, int c, uint32_t vslot_addr, bool acc, bool last) {
        const uint64_t vd = umma_desc_sw128(vslot_addr, kNarrow ? 16 : (kHeadMaps ? 1024 : 16384), kKvSbo);
        for (int q = 0; q < 4; ++q) {
          if (q % 2 == 0) {  // P is published in halves of 64 keys
            if (!mbar_wait(bar(BAR_P_FULL + 2 * t + q / 2), c & 1, abort_flag)) return false;
            tc_fence_after();
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int kk = 2 * q + h;
            // V is the MN-major B operand: 64-column atoms at LBO, 8-key groups at SBO.
            umma_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                    vd + (kv_slot_offset<kHeadMaps, kNarrow>(16 * kk, 0, 0) >> 4), idesc_pv, (acc || kk > 0) ? 1u : 0u);
          }
        }
        if (last) tc_commit(bar(BAR_O_DONE + t));  // the epilogue's wait; earlier tiles need none
        return true;
      };
      auto slot_addr = [&](int g) { return sbase + kSmKV + (g % kKvStages) * 32768; };
      auto wait_full = [&](int g) {
        return mbar_wait(bar(BAR_KV_FULL + g % kKvStages), (g / kKvStages) & 1, abort_flag);
      };
      // head_dim 256: S over the four Q quarters and two K slots; O lo / hi
      // (TMEM columns 256 / 384) from the two V slots, both with P of S0.
      auto issue_s_wide = [&](uint32_t klo, uint32_t khi) {
        const uint64_t qd = umma_desc_sw128(sbase + kSmQ, 16, 1024);
        const uint64_t kdl = umma_desc_sw128(klo, 16, kHeadMaps ? 2048 : 1024);
        const uint64_t kdh = umma_desc_sw128(khi, 16, kHeadMaps ? 2048 : 1024);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t koff = kv_slot_offset<kHeadMaps>(0, (kk >> 2) & 1, 0) + (kk & 3) * 32;
          umma_ss(tmem, qd + (qoff >> 4), (kk < 8 ? kdl : kdh) + (koff >> 4), idesc_qk, kk > 0);
        }
        tc_commit(bar(BAR_S_FULL));
      };
      auto issue_pv_wide = [&](int c, uint32_t vlo, uint32_t vhi, bool acc, bool last) {
        const uint64_t vdl = umma_desc_sw128(vlo, kHeadMaps ? 1024 : 16384, kHeadMaps ? 2048 : 1024);
        const uint64_t vdh = umma_desc_sw128(vhi, kHeadMaps ? 1024 : 16384, kHeadMaps ? 2048 : 1024);
        for (int q = 0; q < 4; ++q) {
          if (q % 2 == 0) {
            if (!mbar_wait(bar(BAR_P_FULL + q / 2), c & 1, abort_flag)) return false;
            tc_fence_after();
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int kk = 2 * q + h;
            const uint32_t voff = kv_slot_offset<kHeadMaps>(16 * kk, 0, 0) >> 4;
            umma_ts(tmem + 256, tmem + kk * 8, vdl + voff, idesc_pv, (acc || kk > 0) ? 1u : 0u);
            umma_ts(tmem + 384, tmem + kk * 8, vdh + voff, idesc_pv, (acc || kk > 0) ? 1u : 0u);
          }
        }
        if (last) tc_commit(bar(BAR_O_DONE));
        return true;
      };
      for (int it = 0; kWide; ++it) {
        // head_dim 256, one query tile per unit: S(j), PV(j), S(j + 1), ...
        // (S(j + 1) overwrites the S columns that hold P(j) only after PV(j)
        // has read them: the tensor core runs them in issue order).
        UnitEntry e;
        if (!take_entry(it, e)) break;
        mbar_arrive(bar(BAR_IT_EMPTY + it % kUnitRing));
        if (!e.valid) break;
        const UnitGeom ug = geometry(e);
        const int n_tiles = ug.n_tiles;
        if (n_tiles == 0) continue;
        bool ok = mbar_wait(bar(BAR_Q_FULL), q_uses & 1, abort_flag);
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int f = fills + 4 * j;
          if (!wait_full(f) || !wait_full(f + 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s_wide(slot_addr(f), slot_addr(f + 1));
          if (j + 1 == n_tiles) tc_commit(bar(BAR_Q_EMPTY));  // the unit's last S is issued
          tc_commit(bar(BAR_KV_EMPTY + f % kKvStages));
          tc_commit(bar(BAR_KV_EMPTY + (f + 1) % kKvStages));
          if (!wait_full(f + 2) || !wait_full(f + 3) ||
              !issue_pv_wide(tiles_done[0] + j, slot_addr(f + 2), slot_addr(f + 3), j > 0, j + 1 == n_tiles)) {
            ok = false;
            break;
          }
          tc_commit(bar(BAR_KV_EMPTY + (f + 2) % kKvStages));
          tc_commit(bar(BAR_KV_EMPTY + (f + 3) % kKvStages));
        }
        if (!ok) break;
        fills += 4 * n_tiles;
        ++q_uses;
        tiles_done[0] += n_tiles;
      }
      for (int it = 0; !kWide; ++it) {
        UnitEntry e;
        if (!take_entry(it, e)) break;
        mbar_arrive(bar(BAR_IT_EMPTY + it % kUnitRing));
        if (!e.valid) break;
        const UnitGeom ug = geometry(e);
        const int n_tiles = ug.n_tiles;
        if (n_tiles == 0) continue;
        const bool two = ug.pos0 + P < ug.q_len;
        bool ok = mbar_wait(bar(BAR_Q_FULL), q_uses & 1, abort_flag) && wait_full(fills);
        if (ok) {
          tc_fence_after();
          issue_s(0, slot_addr(fills));
          if (two) issue_s(1, slot_addr(fills));
          if (n_tiles == 1) tc_commit(bar(BAR_Q_EMPTY));
          tc_commit(bar(BAR_KV_EMPTY + fills % kKvStages));
        }
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int vidx = fills + 2 * j + 1, kidx = fills + 2 * j + 2;
          const bool more = j + 1 < n_tiles;
          if (!wait_full(vidx) || !issue_pv(0, tiles_done[0] + j, slot_addr(vidx), j > 0, !more)) {
            ok = false;
            break;
          }
          if (more) {
            if (!wait_full(kidx)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(0, slot_addr(kidx));
          }
          if (two) {
            if (!issue_pv(1, tiles_done[1] + j, slot_addr(vidx), j > 0, !more)) {
              ok = false;
              break;
            }
            if (more) issue_s(1, slot_addr(kidx));
          }
          if (more && j + 2 == n_tiles) tc_commit(bar(BAR_Q_EMPTY));  // the unit's last S is issued
          tc_commit(bar(BAR_KV_EMPTY + vidx % kKvStages));
          if (more) tc_commit(bar(BAR_KV_EMPTY + kidx % kKvStages));
        }
        if (!ok) break;
        fills += 2 * n_tiles;
        ++q_uses;
        tiles_done[0] += n_tiles;
        if (two) tiles_done[1] += n_tiles;
      }
      // All MMAs issued so far complete before the CTA may free TMEM.
      tc_commit(bar(BAR_DRAIN));
      mbar_wait_drain(bar(BAR_DRAIN), 0);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kAttnSoftmaxRegs));
    // ------------------------------------------------------------ softmax (tile t)
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + t * 128;
    const uint32_t o_addr = tmem + lane_base + 256 + t * 128;
    const float sl2 = a.scale_log2;
    int fills = 0;       // K/V ring fills of the units before this one
    int tiles_done = 0;  // tiles this group processed in earlier units
    int o_units = 0;     // O_DONE phases seen: one per unit with tiles for this group
    bool aborted = false;
    for (int it = 0; !aborted; ++it) {
      UnitEntry e;
      if (!take_entry(it, e)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_IT_EMPTY + it % kUnitRing));
      if (!e.valid) break;
      const UnitGeom ug = geometry(e);
      const int n_tiles = ug.n_tiles;
      const bool two = !kWide && ug.pos0 + P < ug.q_len;
      const int unit_fills = fills;
      fills += kFillsPerTile * n_tiles;
      if (!(t == 0 || two)) continue;
      const int tile_pos0 = ug.pos0 + t * P;
      const int row_pos = tile_pos0 + row / a.group;
      const int row_head = e.kvh * a.group + row % a.group;
      const bool row_valid = row < q_rows && row_pos < ug.q_len;
      const int q_abs = ug.q_abs_min + t * P + row / a.group;
      const int row_hi = min(ug.split_end, q_abs + 1);
      const int unmasked_hi = min(ug.split_end, ug.q_abs_min + t * P + 1);
      // V rows [v_tail_from, v_tail_to) of the last tile: loaded page rows at or past L.
      const int last_start = ug.kv_lo + (n_tiles - 1) * kAttnTileN;
      const int v_tail_from = max(ug.seq_len - last_start, 0);
      const int v_tail_to = min(((ug.kv_hi + kAttnSlice - 1) / kAttnSlice) * kAttnSlice - last_start, kAttnTileN);

      float m_used = -INFINITY;  // running maximum in scaled base-2 units
      float l = 0.f;
      for (int j = 0; j < n_tiles; ++j) {
        const int c = tiles_done + j;
        if (!mbar_wait(bar(BAR_S_FULL + t), c & 1, abort_flag)) {
          aborted = true;
          break;
        }
        __syncwarp();
        tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(s_addr + 32 * c4, sr[c4]);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) tmem_wait_ld(sr[c4]);

        const int tile_start = ug.kv_lo + j * kAttnTileN;
        if (tile_start < ug.split_begin || tile_start + kAttnTileN > unmasked_hi) {
          const int lo = ug.split_begin - tile_start;
          const int hi = row_hi - tile_start;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
            for (int cc = 0; cc < 32; ++cc) {
              const int col = c4 * 32 + cc;
              if (col < lo || col >= hi) sr[c4][cc] = __float_as_uint(-INFINITY);
            }
        }
        // Fast path: when the second half's maximum stays within the rescale
        // threshold of the running maximum, the first half's P is computed
        // against the running maximum at once and checked by its sum (a sum of
        // at most 2^threshold bounds every element the same way), so the
        // first half's maximum pass is skipped.  Any failure in the warp falls
        // back to the full pass, which overwrites the speculative P in TMEM
        // before anything is published; results are identical either way.
        const uint64_t sl2_2 = f2_pack(sl2, sl2);
        uint64_t sum_a = f2_pack(0.f, 0.f), sum_b = sum_a;
        bool fast = false;
        {
          float m1[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c4 = 2; c4 < 4; ++c4)
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
              for (int h = 0; h < 4; ++h)
                m1[k] = fmax3(m1[k], __uint_as_float(sr[c4][8 * h + 2 * k]), __uint_as_float(sr[c4][8 * h + 2 * k + 1]));
          const float mh1 = fmaxf(fmaxf(m1[0], m1[1]), fmaxf(m1[2], m1[3])) * sl2;
          if (__all_sync(0xffffffffu, m_used != -INFINITY && mh1 <= m_used + kRescaleThreshold)) {
            const uint64_t negm_2 = f2_pack(-m_used, -m_used);
#pragma unroll
            for (int c4 = 0; c4 < 2; ++c4) {
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(sr[c4][2 * i]), __uint_as_float(sr[c4][2 * i + 1])), sl2_2, negm_2);
                float x0, x1;
                f2_unpack(x2, x0, x1);
                const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
                if (i & 1) sum_b = f2_add(sum_b, f2_pack(p0, p1)); else sum_a = f2_add(sum_a, f2_pack(p0, p1));
                pk[i] = Pack2<T>::pack(p0, p1);
              }
              tmem_st16(s_addr + 16 * c4, pk);
            }
            float a0, a1;
            f2_unpack(f2_add(sum_a, sum_b), a0, a1);
            fast = __all_sync(0xffffffffu, a0 + a1 <= kRescaleSum);
            if (!fast) sum_a = sum_b = f2_pack(0.f, 0.f);
          }
        }
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
        if (!fast) {
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
          for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              mx[k] = fmax3(mx[k], __uint_as_float(sr[c4][16 * h + 2 * k]), __uint_as_float(sr[c4][16 * h + 2 * k + 1]));
        const float mxa = fmax3(mx[0], mx[1], mx[2]), mxb = fmax3(mx[3], mx[4], mx[5]);
        const float m_cand = fmaxf(m_used, fmax3(mxa, mxb, fmaxf(mx[6], mx[7])) * sl2);
        const bool raise = m_cand > m_used + kRescaleThreshold;  // false while both are -inf
        if (__any_sync(0xffffffffu, raise)) {
          const float alpha = raise ? ex2_approx(m_used - m_cand) : 1.f;  // 0 when m_used = -inf
          if (j > 0) {
            // O holds PV of tiles < j: scale it before PV_j accumulates.  The
            // S_FULL phase of tile j already implies PV_{j-1} is complete: its
            // commit covers every UMMA the issuer started before S_j.
#pragma unroll 1
            for (int c8 = 0; c8 < (kWide ? 16 : kNarrow ? 4 : 8); ++c8) {  // O, 16 columns at a time
              uint32_t o[16];
              tmem_ld16(o_addr + 16 * c8, o);
              tmem_wait_ld16(o);
#pragma unroll
              for (int cc = 0; cc < 16; ++cc) o[cc] = __float_as_uint(__uint_as_float(o[cc]) * alpha);
              tmem_st16(o_addr + 16 * c8, o);
            }
          }
          if (raise) {
            l *= alpha;
            m_used = m_cand;
          }
        }
        }  // !fast
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        if (t == 0 && j == n_tiles - 1 && v_tail_from < v_tail_to) {
          // Rows of the last page past the sequence end may hold anything (NaN
          // included); P is 0 there but 0 * NaN is NaN, so zero those V rows,
          // as the reference's masked V load does (triton_split_kv_paged.py:122).
          bool landed = true;
          for (int vs = 0; vs < (kWide ? 2 : 1) && landed; ++vs) {  // the V slot(s) of the last tile
            const int vidx = unit_fills + kFillsPerTile * j + kFillsPerTile / 2 + vs;
            if (!mbar_wait(bar(BAR_KV_FULL + vidx % kKvStages), (vidx / kKvStages) & 1, abort_flag)) {
              landed = false;
              break;
            }
            const uint32_t vbase = sbase + kSmKV + (vidx % kKvStages) * 32768;
            constexpr int kHalves = kNarrow ? 1 : 2;  // 64-column halves per row in a slot
            const int n16 = (v_tail_to - v_tail_from) * 8 * kHalves;  // 16-byte pieces
            for (int i = threadIdx.x - 128; i < n16; i += 128) {
              const int r = v_tail_from + i / (8 * kHalves);
              const int half = (i >> 3) & (kHalves - 1);
              st_shared_v4(vbase + kv_slot_offset<kHeadMaps, kNarrow>(r, half, i & 7), 0u, 0u, 0u, 0u);
            }
          }
          if (!landed) {
            aborted = true;
            break;
          }
          fence_proxy_async_smem();
        }

        const uint64_t negm_2 = f2_pack(neg_m, neg_m);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t pk[16];
          if (!(fast && c4 < 2)) {  // the fast path has stored quarters 0 and 1 already
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(sr[c4][2 * i]), __uint_as_float(sr[c4][2 * i + 1])), sl2_2, negm_2);
            float x0, x1;
            f2_unpack(x2, x0, x1);
            const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            if (i & 1) sum_b = f2_add(sum_b, f2_pack(p0, p1)); else sum_a = f2_add(sum_a, f2_pack(p0, p1));
            pk[i] = Pack2<T>::pack(p0, p1);
          }
          tmem_st16(s_addr + 16 * c4, pk);
          }
          if (c4 % 2 == 1) {  // publish P in halves: two waits for the issuer per tile instead of four
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(BAR_P_FULL + 2 * t + c4 / 2));  // one arrival per softmax warp
          }
        }
        {
          float a0, a1;
          f2_unpack(f2_add(sum_a, sum_b), a0, a1);
          l += a0 + a1;
        }
      }

      // ---------------------------------------------------------- epilogue
      if (!aborted && n_tiles > 0) {
        if (!mbar_wait(bar(BAR_O_DONE + t), o_units & 1, abort_flag)) aborted = true;
        tc_fence_after();
        ++o_units;
      }
      tiles_done += n_tiles;
      if (aborted) break;
      const float inv = 1.f / fmaxf(l, 1e-20f);
      const int tok = ug.q_begin + row_pos;
      T* dst;
      if (e.nsplit <= 1) {
        dst = static_cast<T*>(a.out) + static_cast<int64_t>(tok) * a.out_st + static_cast<int64_t>(row_head) * a.out_sh;
      } else {
        const int64_t rowi = (static_cast<int64_t>(e.slot) * a.num_splits + e.split) * kUnitRows + t * kAttnTileM + row;
        dst = static_cast<T*>(a.o_split) + rowi * a.head_dim;
        if (row_valid) {
          a.m_split[rowi] = (l > 0.f) ? m_used * 0.69314718055994530942f : -INFINITY;
          a.l_split[rowi] = l;
        }
      }
#pragma unroll
      for (int c4 = 0; c4 < (kWide ? 8 : kNarrow ? 2 : 4); ++c4) {
        if (c4 * 32 >= a.head_dim) break;  // warp-uniform: only the row's real columns
        uint32_t o[32];
        if (n_tiles > 0) {
          tmem_ld32(o_addr + 32 * c4, o);
          tmem_wait_ld(o);
        } else {
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) o[cc] = 0u;
        }
        if (row_valid) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c4 * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = Pack2<T>::pack(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
            w.y = Pack2<T>::pack(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
            w.z = Pack2<T>::pack(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
            w.w = Pack2<T>::pack(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
            d4[v] = w;
          }
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  griddep_launch_dependents();  // the split-unit combine may launch (it waits for this grid to finish)
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Device-side work list, built by one block with no host synchronisation.
//
// Splits: a query unit's split count s is chosen here, at most the caller's
// num_splits.  With W the KV tiles of all (query unit, KV head) pairs, a unit
// of n tiles is split into s = ceil(n * kSplitBalance * SMs / W) runs (at
// least kMinSplitTiles tiles each, none empty): a unit is split only when it
// is more than 1/kSplitBalance of one SM's share of the batch, i.e. when the
// batch is too small to keep every SM busy to the end without it.  The
// uniform mode splits every unit num_splits ways (one run of whole tiles per
// split, none empty), as the reference splits every query block.
//
// Order: sequences by estimated work, heaviest first (a bucket sort on a log
// scale); inside a sequence, query units from the last (most keys) to the
// first, the KV heads and splits of one query unit side by side.  The
// persistent attention CTAs claim units in this order, which is a
// longest-processing-time schedule at sequence granularity (the last
// kSchedThreads units are re-sorted by size across sequences) and keeps the
// CTAs running at any moment on a few sequences, so each sequence's K/V pages
// are read from HBM about once and then served from L2 (ordering units by
// size alone interleaved all sequences and read the 16K workload's K/V from
// HBM six times over).  The unit count and the claim counter stay on the
// device.
// ---------------------------------------------------------------------------
constexpr int kSchedThreads = 1024;
constexpr int kSchedBuckets = 2048;
constexpr float kSchedBucketsPerOctave = 46.0f;  // 2^44 (the largest work estimate) -> bucket 2024
constexpr int kSchedSeqCache = 4096;  // sequences whose arrays the schedule keeps in shared memory
constexpr int kSplitBalance = 2;   // split units larger than half of one SM's share of the batch
constexpr int kMinSplitTiles = 2;  // KV tiles each split keeps at least

struct SchedArgs {
  const void* cu_q;
  const void* seqused;
  int len_i64;
  int num_seqs;
  int pos_per_unit;  // query positions per work unit
  int num_kv_heads;
  int num_splits;    // the most splits a query unit may get
  int uniform_splits;  // 1: every query unit is split num_splits ways
  int num_sms;
  int capacity;
  int* tile_base;    // [num_seqs + 1]: query units per sequence, exclusive prefix
  int* seq_off;      // [num_seqs]: first slot of each sequence's units in the work list
  int* qunit_base;   // [query units + 1]: work units (splits x KV heads) per query unit, exclusive prefix
  int* qunit_split;  // [query units]: splits of each query unit
  int* qunit_slot;   // [query units]: index among the split query units, -1 if not split
  int4* units;
  int4* split_units;  // [split query units x KV heads]: (seq, qunit, kvh, splits), read by the combine
  int* unit_count;    // [0] units, [1] claim counter of the attention kernel, [2] split-unit slots
};

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  total = warp_sums[31];
  __syncthreads();
  return before;
}

// Two exclusive prefix sums over the block in one pass (warp_sums: 64 ints).
__device__ __forceinline__ void block_exclusive_scan2(int v0, int v1, int* warp_sums, int& before0, int& before1,
                                                      int& total0, int& total1) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x0 = v0, x1 = v1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y0 = __shfl_up_sync(0xffffffffu, x0, o);
    const int y1 = __shfl_up_sync(0xffffffffu, x1, o);
    if (lane >= o) {
      x0 += y0;
      x1 += y1;
    }
  }
  if (lane == 31) {
    warp_sums[warp] = x0;
    warp_sums[32 + warp] = x1;
  }
  __syncthreads();
  if (warp == 0) {
    int w0 = warp_sums[lane], w1 = warp_sums[32 + lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y0 = __shfl_up_sync(0xffffffffu, w0, o);
      const int y1 = __shfl_up_sync(0xffffffffu, w1, o);
      if (lane >= o) {
        w0 += y0;
        w1 += y1;
      }
    }
    warp_sums[lane] = w0;  // inclusive over warps
    warp_sums[32 + lane] = w1;
  }
  __syncthreads();
  before0 = (warp > 0 ? warp_sums[warp - 1] : 0) + x0 - v0;
  before1 = (warp > 0 ? warp_sums[32 + warp - 1] : 0) + x1 - v1;
  total0 = warp_sums[31];
  total1 = warp_sums[63];
  __syncthreads();
}

// hist[i] := number of entries in buckets above i (exclusive prefix from the
// top bucket down).
__device__ __forceinline__ void buckets_to_offsets_desc(int* hist, int* warp_sums) {
  constexpr int per = kSchedBuckets / kSchedThreads;
  int local[per];
  int sum = 0;
#pragma unroll
  for (int k = 0; k < per; ++k) {
    local[k] = hist[kSchedBuckets - 1 - (threadIdx.x * per + k)];
    sum += local[k];
  }
  int total;
  int before = block_exclusive_scan(sum, warp_sums, total);
#pragma unroll
  for (int k = 0; k < per; ++k) {
    hist[kSchedBuckets - 1 - (threadIdx.x * per + k)] = before;
    before += local[k];
  }
}

// Last index i in [0, n) with v[i] <= x (v non-decreasing, v[0] <= x).
__device__ __forceinline__ int upper_index(const int* v, int n, int x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (v[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Splits of a query unit whose whole key range has n tiles (see above).
__device__ __forceinline__ int qunit_splits(const SchedArgs& a, int n, long long total_tiles) {
  if (a.num_splits <= 1 || n <= 1) return 1;
  long long s;
  if (a.uniform_splits) {
    s = min(a.num_splits, n);
  } else {
    const long long want = (static_cast<long long>(n) * kSplitBalance * a.num_sms + total_tiles - 1) /
                           max(total_tiles, 1ll);
    s = min(min(static_cast<long long>(a.num_splits), want), static_cast<long long>(n / kMinSplitTiles));
  }
  if (s <= 1) return 1;
  const int tps = (n + static_cast<int>(s) - 1) / static_cast<int>(s);  // whole tiles per split
  return (n + tps - 1) / tps;                                             // no split left empty
}

// Dynamic shared memory of the schedule kernel: the schedule's tail (its
// last kSchedThreads units, re-sorted at the end), the per-sequence arrays
// (query-unit prefix, query length, KV length, first work-list slot) for up
// to kSchedSeqCache sequences and the per-query-unit arrays (splits,
// work-unit prefix, split slot, sequence) for up to kSchedQunitCache query units;
// larger batches keep them in the workspace.  Every pass then reads shared
// memory, and global memory is read once per value.
constexpr int kSchedQunitCache = 8192;
constexpr uint32_t kSchedSmemBytes =
    16 * kSchedThreads + 4 * (kSchedBuckets + 64 + 4 * kSchedSeqCache + 1 + 4 * kSchedQunitCache + 1);

__global__ void __launch_bounds__(kSchedThreads, 1) attn_schedule_kernel(const SchedArgs a) {
  extern __shared__ int4 sched_smem[];
  int4* s_tail = sched_smem;                             // [kSchedThreads]
  int* hist = reinterpret_cast<int*>(s_tail + kSchedThreads);  // [kSchedBuckets]
  int* warp_sums = hist + kSchedBuckets;                 // [64]
  int* s_tb = warp_sums + 64;                            // [kSchedSeqCache + 1]
  int* s_ql = s_tb + kSchedSeqCache + 1;                 // [kSchedSeqCache]
  int* s_L = s_ql + kSchedSeqCache;                      // [kSchedSeqCache]
  int* s_so = s_L + kSchedSeqCache;                      // [kSchedSeqCache]
  int* s_qs = s_so + kSchedSeqCache;                     // [kSchedQunitCache]
  int* s_qb = s_qs + kSchedQunitCache;                   // [kSchedQunitCache + 1]
  int* s_qslot = s_qb + kSchedQunitCache + 1;            // [kSchedQunitCache]
  int* s_qseq = s_qslot + kSchedQunitCache;              // [kSchedQunitCache]
  __shared__ int s_total_qunits;
  __shared__ unsigned long long s_total_tiles;
  griddep_launch_dependents();  // the attention grid may launch; it waits for this one

  const bool seq_cached = a.num_seqs <= kSchedSeqCache;
  auto q_len = [&](int b) {
    return seq_cached ? s_ql[b] : load_index(a.cu_q, b + 1, a.len_i64) - load_index(a.cu_q, b, a.len_i64);
  };
  auto kv_len = [&](int b) { return seq_cached ? s_L[b] : load_index(a.seqused, b, a.len_i64); };

  // 1. query units per sequence, exclusive prefix over sequences.
  int carry = 0;
  for (int base = 0; base < a.num_seqs; base += kSchedThreads) {
    const int b = base + threadIdx.x;
    int n = 0;
    if (b < a.num_seqs) {
      const int ql = load_index(a.cu_q, b + 1, a.len_i64) - load_index(a.cu_q, b, a.len_i64);
      const int L = load_index(a.seqused, b, a.len_i64);
      if (seq_cached) {
        s_ql[b] = ql;
        s_L[b] = L;
      }
      n = ql > 0 ? (ql + a.pos_per_unit - 1) / a.pos_per_unit : 0;
    }
    int total;
    const int before = block_exclusive_scan(n, warp_sums, total);
    if (b < a.num_seqs) {
      a.tile_base[b] = carry + before;
      if (seq_cached) s_tb[b] = carry + before;
    }
    carry += total;
  }
  if (threadIdx.x == 0) {
    a.tile_base[a.num_seqs] = carry;
    if (seq_cached) s_tb[a.num_seqs] = carry;
    s_total_qunits = carry;
    s_total_tiles = 0ull;
  }
  for (int i = threadIdx.x; i < kSchedBuckets; i += kSchedThreads) hist[i] = 0;
  __syncthreads();
  const int nq = s_total_qunits;
  const int* tb = seq_cached ? s_tb : a.tile_base;
  const bool q_cached = nq <= kSchedQunitCache;
  int* qs = q_cached ? s_qs : a.qunit_split;
  int* qb = q_cached ? s_qb : a.qunit_base;
  int* qslot = q_cached ? s_qslot : a.qunit_slot;

  // Each thread takes a contiguous run of query units: one search for the
  // run's first sequence, then a walk along the runs in every pass.
  const int q_per = (nq + kSchedThreads - 1) / kSchedThreads;
  const int j_begin = min(static_cast<int>(threadIdx.x) * q_per, nq);
  const int j_end = min(j_begin + q_per, nq);
  const int seq_begin = j_begin < nq ? upper_index(tb, a.num_seqs, j_begin) : 0;

  // 2. KV tiles of each query unit's whole key range (kept in qs for now) and
  // their sum over query units and KV heads.
  unsigned long long my_tiles = 0;
  for (int j = j_begin, seq = seq_begin; j < j_end; ++j) {
    while (tb[seq + 1] <= j) ++seq;  // past empty sequences
    const int n = qunit_full_tiles(q_len(seq), kv_len(seq), j - tb[seq], a.pos_per_unit);
    qs[j] = n;
    if (q_cached) s_qseq[j] = seq;
    my_tiles += static_cast<unsigned long long>(n);
  }
  if (a.num_splits > 1) {  // one shared atomic per warp (1024 on one word serialise)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) my_tiles += __shfl_xor_sync(0xffffffffu, my_tiles, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s_total_tiles, my_tiles);
  }
  __syncthreads();
  const long long total_tiles = static_cast<long long>(s_total_tiles) * a.num_kv_heads;

  // 3. splits per query unit; work units and split slots, exclusive prefixes
  // (one block scan over the runs' sums).
  int my_units = 0, my_split = 0;
  for (int j = j_begin; j < j_end; ++j) {
    const int sp = qunit_splits(a, qs[j], total_tiles);
    qs[j] = sp;
    my_units += sp * a.num_kv_heads;
    my_split += sp > 1 ? 1 : 0;
  }
  int ubefore, sbefore, ucarry, scarry;
  block_exclusive_scan2(my_units, my_split, warp_sums, ubefore, sbefore, ucarry, scarry);
  for (int j = j_begin; j < j_end; ++j) {
    const int sp = qs[j];
    qb[j] = ubefore;
    qslot[j] = sp > 1 ? sbefore : -1;
    ubefore += sp * a.num_kv_heads;
    sbefore += sp > 1 ? 1 : 0;
  }
  if (threadIdx.x == 0) qb[nq] = ucarry;
  __syncthreads();
  const int total_units = min(ucarry, a.capacity);

  // 4. units per work bucket; each sequence takes a contiguous range of its bucket.
  auto seq_bucket_of = [&](int b, int units) {
    const float keys = fmaxf(static_cast<float>(kv_len(b)) - 0.5f * static_cast<float>(q_len(b)), 1.0f);
    const float work = static_cast<float>(units) * keys;
    return min(kSchedBuckets - 1, max(0, static_cast<int>(__log2f(work) * kSchedBucketsPerOctave)));
  };
  auto seq_units = [&](int b) { return qb[tb[b + 1]] - qb[tb[b]]; };
  for (int b = threadIdx.x; b < a.num_seqs; b += kSchedThreads) {
    const int qt = tb[b + 1] - tb[b];
    if (qt > 0) atomicAdd(&hist[seq_bucket_of(b, qt)], seq_units(b));
  }
  __syncthreads();
  buckets_to_offsets_desc(hist, warp_sums);
  __syncthreads();
  for (int b = threadIdx.x; b < a.num_seqs; b += kSchedThreads) {
    const int qt = tb[b + 1] - tb[b];
    if (qt > 0) {
      const int off = atomicAdd(&hist[seq_bucket_of(b, qt)], seq_units(b));
      a.seq_off[b] = off;
      if (seq_cached) s_so[b] = off;
    }
  }
  __syncthreads();
  const int* so = seq_cached ? s_so : a.seq_off;
  // 5. scatter, one query unit per thread (adjacent threads write adjacent
  // units): a query unit's units (KV head, then split) go to its sequence's
  // range, the sequence's last query unit first.  The units that land in the
  // schedule's tail are also kept in shared memory for step 6.
  const int tail = min(total_units, kSchedThreads);
  const int tail0 = total_units - tail;
  for (int j = threadIdx.x; j < nq; j += kSchedThreads) {
    const int seq = q_cached ? s_qseq[j] : upper_index(tb, a.num_seqs, j);
    const int sp = qs[j];
    const int first = qb[j];
    const int qunit = j - tb[seq];
    const int pos0 = so[seq] + (qb[tb[seq + 1]] - qb[j + 1]);
    const int slot0 = sp > 1 ? qslot[j] * a.num_kv_heads : -1;
    for (int rem = 0; rem < sp * a.num_kv_heads && first + rem < total_units; ++rem) {
      const int kvh = rem / sp;
      const int split = rem - kvh * sp;
      const int slot = sp > 1 ? slot0 + kvh : -1;
      const int pos = pos0 + rem;
      const int4 u = pack_unit(seq, qunit, kvh, split, sp, slot);
      if (pos < a.capacity) a.units[pos] = u;
      if (pos >= tail0 && pos < total_units) s_tail[pos - tail0] = u;
      if (sp > 1 && split == 0) a.split_units[slot] = make_int4(seq, qunit, kvh, sp);
    }
  }
  __syncthreads();
  // 6. the schedule's tail, its last kSchedThreads units, by KV-tile count
  // across sequences, heaviest first, so the last units claimed are the
  // smallest.
  const bool mine = static_cast<int>(threadIdx.x) < tail;
  int4 unit = make_int4(0, 0, 0, 0);
  int bucket = 0;
  if (mine) {
    // Every tail slot was written in step 5 unless the capacity clipped the list.
    unit = ucarry == total_units ? s_tail[threadIdx.x] : a.units[tail0 + threadIdx.x];
    int kvh, split, nsplit;
    unpack_unit(unit, kvh, split, nsplit);
    const int q0 = seq_cached ? 0 : load_index(a.cu_q, unit.x, a.len_i64);
    const UnitGeom g = unit_geometry(q0, q0 + q_len(unit.x), kv_len(unit.x), unit.y, split, nsplit, a.pos_per_unit);
    bucket = min(g.n_tiles, kSchedBuckets - 1);
  }
  for (int i = threadIdx.x; i < kSchedBuckets; i += kSchedThreads) hist[i] = 0;
  __syncthreads();
  if (mine) atomicAdd(&hist[bucket], 1);
  __syncthreads();
  buckets_to_offsets_desc(hist, warp_sums);
  __syncthreads();
  if (mine) a.units[tail0 + atomicAdd(&hist[bucket], 1)] = unit;
  if (threadIdx.x == 0) {
    a.unit_count[0] = total_units;
    a.unit_count[1] = 0;  // claim counter of the persistent attention kernel
    a.unit_count[2] = scarry * a.num_kv_heads;  // split-unit slots for the combine
  }
}

// ---------------------------------------------------------------------------
// Combine of the split units' partials: one (token, head) row of a split unit
// per D/8 threads, over a grid-stride loop whose bound (the split-unit count)
// the schedule kernel left on the device; a call without split units costs
// one launch that exits at once.  Row r of a unit is query tile r / 128, tile
// row r % 128 = (position, head) as in the attention kernel; padding rows,
// tiles the unit does not have and positions past the sequence's query rows
// are skipped.
// ---------------------------------------------------------------------------
struct UnitCombineArgs {
  const void* o_part;      // [slots][num_splits][kUnitRows][head_dim], query dtype
  const float* m_part;     // [slots][num_splits][kUnitRows]
  const float* l_part;
  const int4* split_units;
  const int* unit_count;   // [2] = slots
  const void* cu_q;
  void* out;
  int64_t out_st, out_sh;
  int len_i64;
  int num_splits;
  int group;
  int pos_per_tile;
  int pos_per_unit;
};

template <typename T, int D, int kS>
__global__ void __launch_bounds__(kCombineThreads) unit_combine_kernel(const UnitCombineArgs a) {
  constexpr int kThreadsPerRow = D / 8;
  constexpr int kRowsPerBlock = kCombineThreads / kThreadsPerRow;
  griddep_wait();  // launched as a programmatic dependent of the attention kernel
  const int64_t rows = static_cast<int64_t>(a.unit_count[2]) * kUnitRows;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock; base < rows;
       base += static_cast<int64_t>(gridDim.x) * kRowsPerBlock) {
    const int64_t row_raw = base + threadIdx.x / kThreadsPerRow;
    const bool in_range = row_raw < rows;  // threads past the end still take part in the shuffles
    const int64_t row = in_range ? row_raw : rows - 1;
    const int slot = static_cast<int>(row / kUnitRows);
    const int ur = static_cast<int>(row - static_cast<int64_t>(slot) * kUnitRows);
    const int4 su = a.split_units[slot];  // (seq, qunit, kvh, splits)
    const int t = ur / kAttnTileM, r = ur % kAttnTileM;
    const int q_begin = load_index(a.cu_q, su.x, a.len_i64);
    const int q_len = load_index(a.cu_q, su.x + 1, a.len_i64) - q_begin;
    const int pos = su.y * a.pos_per_unit + t * a.pos_per_tile + r / a.group;
    // Rows of a tile the unit does not have (the second tile of a head_dim-256
    // unit, which holds one) would name the next unit's positions: skipped.
    const bool valid = in_range && r < a.group * a.pos_per_tile && t * a.pos_per_tile < a.pos_per_unit && pos < q_len;
    const int64_t prow = static_cast<int64_t>(slot) * a.num_splits * kUnitRows + ur;
    const int64_t tok = q_begin + pos, head = static_cast<int64_t>(su.z) * a.group + r % a.group;
    combine_row<T, T, D, kS>(static_cast<const T*>(a.o_part) + prow * D, static_cast<int64_t>(kUnitRows) * D,
                             a.m_part + prow, kUnitRows, a.l_part + prow, kUnitRows, su.w,
                             static_cast<T*>(a.out) + tok * a.out_st + head * a.out_sh, valid);
  }
}

}  // namespace b200
