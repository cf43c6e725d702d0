// paged_decode.cuh -- paged attention for decode batches (every sequence has
// one query token) on sm_100a.
//
// Same result as the Split-KV kernel for such a batch (the query token of
// sequence b sits at position L_b - 1 and sees keys [0, L_b); GQA: query head
// h reads KV head h / G): softmax(q K^T * scale) V over the sequence, in fp32,
// stored in the query dtype.  A sequence with L_b = 0 gets zeros.
//
// Decode streams every K/V row once for only G query rows per KV head, so the
// bound is HBM bandwidth and the layout is chosen for it:
//   * work item = (sequence, KV head, chunk of C keys); the schedule kernel
//     lists the items longest first and persistent CTAs claim them from a
//     global counter (the producer of K claims, and hands the item to the
//     other warps through a 4-entry ring in shared memory), so the CTAs end
//     within about one item of each other and the K/V rings keep streaming
//     across item boundaries; each item leaves a partial (unnormalised O, m, l)
//     that decode_combine_kernel merges per (sequence, query head);
//   * the UMMAs put the keys on M: S^T = K_j Q^T (M = 128 keys, N = 16 query
//     heads of the group padded with zero rows, K = head_dim), and
//     O^T += V_j^T P^T (M = head_dim, N = 16, K = 128 keys; V^T is the V tile
//     read MN-major).  The tensor core does 16 x the needed work, which is
//     still far below the time the tile takes to arrive.
// Warps: 0 TMA producer of Q (per item) and K_j, 2 TMA producer of V_j (K and
// V tiles of 128 keys, each through its own 3-slot ring of 32 KB), 1 UMMA
// issuer and TMEM owner, 4..7 softmax: thread r
// holds key r of the tile (S^T row r) and, for the O rescale and the
// epilogue, row d = r of O^T.  The per-head maxima over the tile's 128 keys
// are butterfly reductions in each warp, exchanged through shared memory
// under an mbarrier; the running maximum is raised only when it grows by more
// than 2^8 (then O^T is rescaled); row sums stay per thread until the item
// ends.  P^T (bf16 / f16) is written to shared memory in the UMMA's K-major
// 128-byte-swizzled layout.
// K/V tile layout: one TMA box per page slice of 16 keys brings both 64-column
// halves of head_dim (a 5-D map per KV head: d, key % 8, half, key / 8 in the
// page, page), so a tile is 16 groups of 8 keys at 2 KB strides, each group
// holding half 0 then half 1 as 1 KB swizzle atoms.  Page lookups run one
// tile ahead of the copies; lane c of a producer warp owns slice c.
#pragma once

#include "paged_attention.cuh"

namespace b200 {

constexpr int kDecThreads = 256;
constexpr int kDecTileN = 128;     // keys per tile (UMMA M of S^T)
constexpr int kDecN = 16;          // UMMA N: query heads of a group, zero-padded
constexpr int kDecStages = 3;      // slots of 32 KB in each of the K and V rings
constexpr int kDecMaxKvHeads = kMaxHeadMaps;  // per-head tensor maps passed as kernel parameters
constexpr int kDecTmemCols = 64;   // S^T ring 2 x 16 columns, O^T 2 x 16 columns
constexpr float kDecRescale = 8.0f;

constexpr uint32_t kDsQ = 0;                                // 2 x 4 KB: two d-halves of 16 rows x 128 B
constexpr uint32_t kDsP = 8192;                             // 2 x 4 KB: two key-halves of 16 rows x 128 B
constexpr uint32_t kDsK = 16384;                            // K ring
constexpr uint32_t kDsV = kDsK + kDecStages * 32768;        // V ring
constexpr uint32_t kDsRed = kDsV + kDecStages * 32768;      // 2 x 4 x 16 floats (max), 4 x 16 floats (sum)
constexpr uint32_t kDsItems = kDsRed + 768;                 // ring of claimed items (8 ints each)
constexpr int kDecItemRing = 4;
constexpr uint32_t kDsBar = kDsRed + 1024;
constexpr uint32_t kDsBytes = kDsBar + 512;
constexpr uint32_t kDecodeSmemAlloc = kDsBytes + 1024;

enum : int {
  DB_Q_FULL = 0,    // + buffer
  DB_Q_EMPTY = 2,   // + buffer
  DB_K_FULL = 4,    // + slot
  DB_K_EMPTY = DB_K_FULL + kDecStages,
  DB_V_FULL = DB_K_EMPTY + kDecStages,
  DB_V_EMPTY = DB_V_FULL + kDecStages,
  DB_S_FULL = DB_V_EMPTY + kDecStages,   // + buffer
  DB_P_FULL = DB_S_FULL + 2,             // + buffer, 4 arrivals
  DB_P_EMPTY = DB_P_FULL + 2,            // + buffer: the P^T V UMMAs of the buffer's tile are done
  DB_O_FREE = DB_P_EMPTY + 2,            // + buffer, 4 arrivals
  DB_RED = DB_O_FREE + 2,                // + buffer, 4 arrivals
  DB_LRED = DB_RED + 2,                  // 4 arrivals
  DB_IT_FULL = DB_LRED + 1,              // + ring entry
  DB_IT_EMPTY = DB_IT_FULL + kDecItemRing,  // + ring entry, 6 arrivals (V producer, UMMA, 4 softmax warps)
  DB_DRAIN = DB_IT_EMPTY + kDecItemRing,
  DB_COUNT = DB_DRAIN + 1
};
static_assert(DB_COUNT * 8 + 8 <= 512, "barrier area");

struct DecodeArgs {
  const void* block_table;
  const void* cu_q;
  const void* seqused;
  int* item_base;  // [num_seqs + 2]: first item of each sequence, total, claim counter
  int* order;      // [items]: item indices, longest first
  float* part_o;   // [items][G][128], unnormalised
  float* part_m;   // [items][G], running maximum in scaled base-2 units
  float* part_l;   // [items][G]
  int64_t bt_stride;
  int bt_cols, bt_i64, len_i64;
  int num_seqs, num_kv_heads;
  int chunk;  // keys per item, a multiple of 128
  int block_size, num_blocks;
  float scale_log2;
};

// One 5-D tensor map per KV head for each of K and V (see the header comment).
using DecodeMaps = KvHeadMaps;

struct DecodeItem {
  int seq, kvh, kv_begin, kv_end, L, n_tiles;
};

// `base` is item_base (global memory) or a copy of it in shared memory.
__device__ __forceinline__ DecodeItem decode_item(const DecodeArgs& a, const int* base, int item) {
  int lo = 0, hi = a.num_seqs - 1;  // last sequence whose first item is <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (base[mid] <= item) lo = mid; else hi = mid - 1;
  }
  DecodeItem d;
  d.seq = lo;
  d.L = load_index(a.seqused, lo, a.len_i64);
  const int chunks = (d.L + a.chunk - 1) / a.chunk;
  const int rem = item - base[lo];
  d.kvh = rem / chunks;
  d.kv_begin = (rem - d.kvh * chunks) * a.chunk;
  d.kv_end = min(d.kv_begin + a.chunk, d.L);
  d.n_tiles = (d.kv_end - d.kv_begin + kDecTileN - 1) / kDecTileN;
  return d;
}

// Items per sequence (KH x chunks of its keys; none unless it has exactly one
// query token and at least one key), exclusive prefix into item_base; then the
// item list ordered by tile count, longest first (bucket sort), and the claim
// counter reset.
constexpr int kDecSchedSmemSeqs = 4096;  // item_base kept in shared memory up to this many sequences

__global__ void __launch_bounds__(kSchedThreads, 1) decode_schedule_kernel(const DecodeArgs a) {
  __shared__ int warp_sums[32];
  __shared__ int hist[kSchedBuckets];
  __shared__ int s_base[kDecSchedSmemSeqs + 1];
  __shared__ int s_total;
  const bool in_smem = a.num_seqs <= kDecSchedSmemSeqs;
  // The decode kernel may launch now: it sets itself up and then waits for
  // this grid before it reads the item list.
  griddep_launch_dependents();
  int carry = 0;
  for (int base = 0; base < a.num_seqs; base += kSchedThreads) {
    const int b = base + threadIdx.x;
    int n = 0;
    if (b < a.num_seqs) {
      const int ql = load_index(a.cu_q, b + 1, a.len_i64) - load_index(a.cu_q, b, a.len_i64);
      const int L = load_index(a.seqused, b, a.len_i64);
      if (ql > 1) record_device_error(B200_DEVERR_DECODE_QLEN);
      n = (ql == 1 && L > 0) ? a.num_kv_heads * ((L + a.chunk - 1) / a.chunk) : 0;
    }
    int total;
    const int before = block_exclusive_scan(n, warp_sums, total);
    if (b < a.num_seqs) {
      a.item_base[b] = carry + before;
      if (in_smem) s_base[b] = carry + before;
    }
    carry += total;
  }
  if (threadIdx.x == 0) {
    a.item_base[a.num_seqs] = carry;
    a.item_base[a.num_seqs + 1] = 0;
    s_total = carry;
  }
  for (int i = threadIdx.x; i < kSchedBuckets; i += kSchedThreads) hist[i] = 0;
  __syncthreads();
  const int total = s_total;
  const int* base = in_smem ? s_base : a.item_base;
  auto bucket_of = [&](int item) { return min(decode_item(a, base, item).n_tiles, kSchedBuckets - 1); };
  for (int u = threadIdx.x; u < total; u += kSchedThreads) atomicAdd(&hist[bucket_of(u)], 1);
  __syncthreads();
  buckets_to_offsets_desc(hist, warp_sums);
  __syncthreads();
  for (int u = threadIdx.x; u < total; u += kSchedThreads) a.order[atomicAdd(&hist[bucket_of(u)], 1)] = u;
}

// Byte offset of element (row, col) of a [16 x 128] bf16/f16 operand stored
// K-major with 128-byte swizzle as two 64-column halves of 2 KB.
__device__ __forceinline__ uint32_t sw128_offset_16x128(int row, int col) {
  const int half = col >> 6, c = col & 63;
  return half * 2048 + (row >> 3) * 1024 + (row & 7) * 128 + ((((c >> 3) ^ (row & 7)) & 7) << 4) + (c & 7) * 2;
}

template <typename T>
__device__ __forceinline__ void st_shared_u16(uint32_t addr, T v) {
  const uint16_t bits = *reinterpret_cast<const uint16_t*>(&v);
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(bits) : "memory");
}

template <typename T>
__device__ __forceinline__ T to_storage(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 to_storage<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half to_storage<__half>(float x) { return __float2half_rn(x); }

// Offset of key row t (0..127), byte b (0..255) of head_dim, inside a K/V tile.
__device__ __forceinline__ uint32_t kv_tile_row_offset(int t, int half) {
  return (t >> 3) * 2048 + half * 1024 + (t & 7) * 128;
}

template <typename T, int G>
__global__ void __launch_bounds__(kDecThreads, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ DecodeMaps maps,
                        const DecodeArgs a) {
  static_assert(G >= 1 && G <= kDecN, "query heads per KV head");
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDsBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kDsBar + DB_COUNT * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kDsBar + DB_COUNT * 8 + 4);
  float* red = reinterpret_cast<float*>(smem + kDsRed);  // [2][4][16] maxima, then [4][16] sums
  // Ring entry: {item, seq, kvh, kv_begin, kv_end, L, n_tiles, -}.
  volatile int* item_ring = reinterpret_cast<volatile int*>(smem + kDsItems);
  auto bar = [&](int i) { return smem_addr(&bars[i]); };
  // Item n of this CTA, as claimed and decoded by the K producer; -1 ends the
  // loop (also on abort).  Lane 0 waits; the warp reads the entry.
  auto pop_item = [&](int n, DecodeItem& d) -> int {
    const int e = n % kDecItemRing;
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar(DB_IT_FULL + e), (n / kDecItemRing) & 1, abort_flag);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    const volatile int* en = item_ring + 8 * e;
    const int item = ok ? en[0] : -1;
    d.seq = en[1];
    d.kvh = en[2];
    d.kv_begin = en[3];
    d.kv_end = en[4];
    d.L = en[5];
    d.n_tiles = en[6];
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar(DB_IT_EMPTY + e));
    return item;
  };
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(DB_Q_FULL + b), 1);
      mbar_init(bar(DB_Q_EMPTY + b), 1);
      mbar_init(bar(DB_S_FULL + b), 1);
      mbar_init(bar(DB_P_FULL + b), 4);
      mbar_init(bar(DB_P_EMPTY + b), 1);
      mbar_init(bar(DB_O_FREE + b), 4);
      mbar_init(bar(DB_RED + b), 4);
    }
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(bar(DB_K_FULL + s), 1);
      mbar_init(bar(DB_K_EMPTY + s), 1);
      mbar_init(bar(DB_V_FULL + s), 1);
      mbar_init(bar(DB_V_EMPTY + s), 1);
    }
    mbar_init(bar(DB_LRED), 4);
    for (int e = 0; e < kDecItemRing; ++e) {
      mbar_init(bar(DB_IT_FULL + e), 1);
      mbar_init(bar(DB_IT_EMPTY + e), 6);
    }
    mbar_init(bar(DB_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Q and P^T buffers start at zero: rows G..15 stay zero (the padded heads).
  for (int i = threadIdx.x; i < 16384 / 16; i += kDecThreads) st_shared_v4(sbase + kDsQ + i * 16, 0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), kDecTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Set-up done; the item list of the schedule kernel is needed from here on.
  griddep_wait();
  const int total = a.item_base[a.num_seqs];

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ producers (whole warps)
    // Warp 0 loads Q and the K tiles, warp 2 the V tiles; lane c < 8 looks up
    // and copies page slice c (16 keys, both halves of head_dim) of each tile.
    const bool is_k = warp == 0;
    const uint32_t ring = sbase + (is_k ? kDsK : kDsV);
    const int full0 = is_k ? DB_K_FULL : DB_V_FULL, empty0 = is_k ? DB_K_EMPTY : DB_V_EMPTY;
    if (lane == 0) {
      if (is_k) tma_prefetch_desc(&tm_q);
      for (int h = 0; h < a.num_kv_heads; ++h) tma_prefetch_desc(is_k ? &maps.k[h] : &maps.v[h]);
    }
    // Physical page and in-page offset of slice (lane & 7) of tile j; slices
    // past the item's last key get page num_blocks, which TMA turns into zeros.
    auto lookup = [&](const DecodeItem& d, int j, int& pg, int& of) {
      const int pos = d.kv_begin + j * kDecTileN + (lane & 7) * kAttnSlice;
      const int lp = pos / a.block_size;
      of = pos - lp * a.block_size;
      const int v = load_index(a.block_table, static_cast<int64_t>(d.seq) * a.bt_stride + min(lp, a.bt_cols - 1),
                               a.bt_i64);
      pg = (pos < d.kv_end && lp < a.bt_cols) ? v : a.num_blocks;
    };
    int fills = 0, q_uses0 = 0, q_uses1 = 0;
    bool ok = true;
    int* counter = a.item_base + a.num_seqs + 1;
    int claimed = -1;
    if (is_k && lane == 0) {
      const int k = atomicAdd(counter, 1);
      claimed = k < total ? a.order[k] : -1;
    }
    for (int it = 0; ok; ++it) {
      int item;
      DecodeItem d{};
      if (is_k) {
        // Decode and publish the claimed item to the other warps, then claim
        // the next one (its latency overlaps this item's copies).
        int okr = 1;
        if (lane == 0) {
          const int e = it % kDecItemRing;
          okr = mbar_wait(bar(DB_IT_EMPTY + e), ((it / kDecItemRing) & 1) ^ 1, abort_flag);
          if (okr && claimed >= 0) d = decode_item(a, a.item_base, claimed);
          volatile int* en = item_ring + 8 * e;
          en[0] = okr ? claimed : -1;
          en[1] = d.seq;
          en[2] = d.kvh;
          en[3] = d.kv_begin;
          en[4] = d.kv_end;
          en[5] = d.L;
          en[6] = d.n_tiles;
          mbar_arrive(bar(DB_IT_FULL + e));
        }
        item = __shfl_sync(0xffffffffu, okr ? claimed : -1, 0);
        d.seq = __shfl_sync(0xffffffffu, d.seq, 0);
        d.kvh = __shfl_sync(0xffffffffu, d.kvh, 0);
        d.kv_begin = __shfl_sync(0xffffffffu, d.kv_begin, 0);
        d.kv_end = __shfl_sync(0xffffffffu, d.kv_end, 0);
        d.L = __shfl_sync(0xffffffffu, d.L, 0);
        d.n_tiles = __shfl_sync(0xffffffffu, d.n_tiles, 0);
        if (item >= 0 && lane == 0) {
          const int k = atomicAdd(counter, 1);
          claimed = k < total ? a.order[k] : -1;
        }
      } else {
        item = pop_item(it, d);
      }
      if (item < 0) break;
      const CUtensorMap* map = is_k ? &maps.k[d.kvh] : &maps.v[d.kvh];
      int pg_cur, of_cur, pg_nxt = a.num_blocks, of_nxt = 0;
      lookup(d, 0, pg_cur, of_cur);
      if (is_k) {
        const int qb = it & 1;
        int okq = 1;
        if (lane == 0) {
          okq = mbar_wait(bar(DB_Q_EMPTY + qb), ((it >> 1) & 1) ^ 1, abort_flag);
          if (okq) {
            const int tok = load_index(a.cu_q, d.seq, a.len_i64);
            mbar_arrive_expect_tx(bar(DB_Q_FULL + qb), 2 * G * 128);
            tma_load_3d(sbase + kDsQ + qb * 4096, &tm_q, bar(DB_Q_FULL + qb), 0, d.kvh * G, tok);
            tma_load_3d(sbase + kDsQ + qb * 4096 + 2048, &tm_q, bar(DB_Q_FULL + qb), 64, d.kvh * G, tok);
          }
        }
        if (!__shfl_sync(0xffffffffu, okq, 0)) break;
        if (qb) ++q_uses1; else ++q_uses0;
      }
      for (int j = 0; j < d.n_tiles; ++j) {
        if (j + 1 < d.n_tiles) lookup(d, j + 1, pg_nxt, of_nxt);
        const int slot = fills % kDecStages;
        int okl = 1;
        if (lane == 0) {
          okl = mbar_wait(bar(empty0 + slot), ((fills / kDecStages) & 1) ^ 1, abort_flag);
          if (okl) mbar_arrive_expect_tx(bar(full0 + slot), 32768);
        }
        if (!__shfl_sync(0xffffffffu, okl, 0)) {
          ok = false;
          break;
        }
        if (lane < 8) tma_load_5d(ring + slot * 32768 + lane * 4096, map, bar(full0 + slot), 0, 0, 0, of_cur >> 3, pg_cur);
        ++fills;
        pg_cur = pg_nxt;
        of_cur = of_nxt;
      }
    }
    // Tail: every issued copy lands, and the UMMA commits that release the
    // slots arrive, before this CTA's shared memory can be reused.
    if (lane == 0) {
      if (q_uses0 > 0) mbar_wait_drain(bar(DB_Q_FULL + 0), (q_uses0 - 1) & 1);
      if (q_uses1 > 0) mbar_wait_drain(bar(DB_Q_FULL + 1), (q_uses1 - 1) & 1);
      for (int s = 0; s < kDecStages && s < fills; ++s) {
        const int last_idx = s + kDecStages * ((fills - 1 - s) / kDecStages);
        const uint32_t last = (last_idx / kDecStages) & 1;
        mbar_wait_drain(bar(full0 + s), last);
        if (!*abort_flag) mbar_wait_drain(bar(empty0 + s), last);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(kBF16, 128, kDecN, false, false);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBF16, 128, kDecN, true, false);
      struct Pending {
        int vidx, it, tile;
        bool first, valid;
      } pend{0, 0, 0, false, false};
      // O^T += V^T P^T for a tile whose P^T the softmax warps have published.
      auto issue_pv = [&](const Pending& p) -> bool {
        if (!mbar_wait(bar(DB_P_FULL + (p.tile & 1)), (p.tile >> 1) & 1, abort_flag)) return false;
        if (!mbar_wait(bar(DB_V_FULL + p.vidx % kDecStages), (p.vidx / kDecStages) & 1, abort_flag)) return false;
        if (p.first && !mbar_wait(bar(DB_O_FREE + (p.it & 1)), ((p.it >> 1) & 1) ^ 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t vaddr = sbase + kDsV + (p.vidx % kDecStages) * 32768;
        const uint32_t paddr = sbase + kDsP + (p.tile & 1) * 4096;
        // A = V^T, MN-major: 64-element d atoms 1 KB apart, 8-key groups 2 KB apart.
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss(tmem + 32 + (p.it & 1) * 16, umma_desc_sw128(vaddr + kk * 4096, 1024, 2048),
                  umma_desc_sw128(paddr + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), idesc_o,
                  (!p.first || kk > 0) ? 1u : 0u);
        tc_commit(bar(DB_V_EMPTY + p.vidx % kDecStages));
        tc_commit(bar(DB_P_EMPTY + (p.tile & 1)));
        return true;
      };
      int tile = 0;  // tile = index of the K fill and of the V fill
      bool ok = true;
      for (int it = 0; ok; ++it) {
        int item = -1;
        DecodeItem d{};
        {
          const int e = it % kDecItemRing;
          if (mbar_wait(bar(DB_IT_FULL + e), (it / kDecItemRing) & 1, abort_flag)) item = item_ring[8 * e];
          d.n_tiles = item_ring[8 * e + 6];
          mbar_arrive(bar(DB_IT_EMPTY + e));
        }
        if (item < 0) break;
        const int qb = it & 1;
        if (!mbar_wait(bar(DB_Q_FULL + qb), (it >> 1) & 1, abort_flag)) break;
        for (int j = 0; j < d.n_tiles; ++j, ++tile) {
          const int kidx = tile, vidx = tile;
          if (!mbar_wait(bar(DB_K_FULL + kidx % kDecStages), (kidx / kDecStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kaddr = sbase + kDsK + (kidx % kDecStages) * 32768;
          const uint32_t qaddr = sbase + kDsQ + qb * 4096;
          // A = K, K-major: half h of head_dim at +1 KB, 8-key groups 2 KB apart.
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_ss(tmem + (tile & 1) * 16, umma_desc_sw128(kaddr + (kk >> 2) * 1024 + (kk & 3) * 32, 16, 2048),
                    umma_desc_sw128(qaddr + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          tc_commit(bar(DB_S_FULL + (tile & 1)));
          tc_commit(bar(DB_K_EMPTY + kidx % kDecStages));
          if (j + 1 == d.n_tiles) tc_commit(bar(DB_Q_EMPTY + qb));
          if (pend.valid && !issue_pv(pend)) {
            ok = false;
            break;
          }
          pend = Pending{vidx, it, tile, j == 0, true};
          // The item's last P^T V goes out at once: its epilogue waits for it,
          // and nothing of the next item may overtake it.
          if (j + 1 == d.n_tiles) {
            if (!issue_pv(pend)) {
              ok = false;
              break;
            }
            pend.valid = false;
          }
        }
      }

      tc_commit(bar(DB_DRAIN));
      mbar_wait_drain(bar(DB_DRAIN), 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    // Parity waits on P_EMPTY[t & 1] (phases: the P^T V groups of tiles t,
    // t + 2, ...) are unambiguous here: a group two tiles later needs this
    // warpgroup's next P^T first, and the group two tiles earlier was already
    // awaited before P^T of tile t was written.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row of S^T; row d of O^T
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = a.scale_log2;
    int tile = 0;
    bool aborted = false;
    for (int it = 0; !aborted; ++it) {
      DecodeItem d{};
      const int item = pop_item(it, d);
      if (item < 0) break;
      float m_used[G], l_thr[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        m_used[h] = -INFINITY;
        l_thr[h] = 0.f;
      }
      const uint32_t o_addr = tmem + lane_base + 32 + (it & 1) * 16;
      for (int j = 0; j < d.n_tiles; ++j, ++tile) {
        const int sb = tile & 1;
        if (!mbar_wait(bar(DB_S_FULL + sb), (tile >> 1) & 1, abort_flag)) {
          aborted = true;
          break;
        }
        __syncwarp();
        tc_fence_after();
        uint32_t s[16];
        tmem_ld16(tmem + lane_base + sb * 16, s);
        tmem_wait_ld16(s);
        const int tile_start = d.kv_begin + j * kDecTileN;
        const bool valid = tile_start + r < d.kv_end;
        float x[G], mx[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          x[h] = valid ? __uint_as_float(s[h]) : -INFINITY;
          mx[h] = x[h];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
          for (int h = 0; h < G; ++h) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
        float* rbuf = red + sb * 64;
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < G; ++h) rbuf[quarter * 16 + h] = mx[h];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(DB_RED + sb));
        if (!mbar_wait(bar(DB_RED + sb), (tile >> 1) & 1, abort_flag)) {
          aborted = true;
          break;
        }
        bool raise_any = false;
        float m_cand[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float mt = fmaxf(fmaxf(rbuf[h], rbuf[16 + h]), fmaxf(rbuf[32 + h], rbuf[48 + h]));
          m_cand[h] = fmaxf(m_used[h], mt * sl2);
          raise_any |= m_cand[h] > m_used[h] + kDecRescale;
        }
        if (raise_any) {  // the same decision in every softmax thread
          float alpha[G];
#pragma unroll
          for (int h = 0; h < G; ++h) alpha[h] = (m_cand[h] > m_used[h] + kDecRescale) ? ex2_approx(m_used[h] - m_cand[h]) : 1.f;
          if (j > 0) {
            // O^T holds the earlier tiles of this item: scale it once their
            // UMMAs are done (the P^T buffer of tile - 1 is released by them),
            // before PV_j.
            if (!mbar_wait(bar(DB_P_EMPTY + ((tile - 1) & 1)), ((tile - 1) >> 1) & 1, abort_flag)) {
              aborted = true;
              break;
            }
            tc_fence_after();
            uint32_t o[16];
            tmem_ld16(o_addr, o);
            tmem_wait_ld16(o);
#pragma unroll
            for (int h = 0; h < G; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
            tmem_st16(o_addr, o);
            tmem_wait_st();
          }
#pragma unroll
          for (int h = 0; h < G; ++h)
            if (m_cand[h] > m_used[h] + kDecRescale) {
              l_thr[h] *= alpha[h];
              m_used[h] = m_cand[h];
            }
        }
        // Rows of the last page past the sequence end may hold anything (NaN
        // included); P is 0 there but 0 * NaN is NaN, so zero those V rows.
        if (d.kv_end == d.L && tile_start + kDecTileN > d.L && (d.L & (kAttnSlice - 1))) {
          if (!mbar_wait(bar(DB_V_FULL + tile % kDecStages), (tile / kDecStages) & 1, abort_flag)) {
            aborted = true;
            break;
          }
          const uint32_t vbase = sbase + kDsV + (tile % kDecStages) * 32768;
          const int from = d.L - tile_start, to = ((d.L + kAttnSlice - 1) / kAttnSlice) * kAttnSlice - tile_start;
          for (int i = r; i < (to - from) * 16; i += 128) {
            const int row = from + (i >> 4);
            st_shared_v4(vbase + kv_tile_row_offset(row, (i >> 3) & 1) + (i & 7) * 16, 0u, 0u, 0u, 0u);
          }
        }
        // P^T row h, column r.
        if (!mbar_wait(bar(DB_P_EMPTY + sb), ((tile >> 1) & 1) ^ 1, abort_flag)) {
          aborted = true;
          break;
        }
        const uint32_t pbuf = sbase + kDsP + sb * 4096;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float p = valid ? ex2_approx(x[h] * sl2 - m_used[h]) : 0.f;
          l_thr[h] += p;
          st_shared_u16<T>(pbuf + sw128_offset_16x128(h, r), to_storage<T>(p));
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(DB_P_FULL + sb));
      }
      if (aborted) break;

      // ---------------------------------------------------------- item epilogue
      float l[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float v = l_thr[h];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        l[h] = v;
      }
      float* lbuf = red + 128;
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < G; ++h) lbuf[quarter * 16 + h] = l[h];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(DB_LRED));
      // The item's last P^T V group is done (UMMAs complete in issue order).
      if (!mbar_wait(bar(DB_P_EMPTY + ((tile - 1) & 1)), ((tile - 1) >> 1) & 1, abort_flag) ||
          !mbar_wait(bar(DB_LRED), it & 1, abort_flag)) {
        aborted = true;
        break;
      }
      tc_fence_after();
      uint32_t o[16];
      tmem_ld16(o_addr, o);
      tmem_wait_ld16(o);
      float* po = a.part_o + static_cast<int64_t>(item) * G * 128;
#pragma unroll
      for (int h = 0; h < G; ++h) po[h * 128 + r] = __uint_as_float(o[h]);
      if (quarter == 0 && lane < G) {
        float mv = 0.f, lv = 0.f;
#pragma unroll
        for (int h = 0; h < G; ++h)
          if (h == lane) {
            mv = m_used[h];
            lv = lbuf[h] + lbuf[16 + h] + lbuf[32 + h] + lbuf[48 + h];
          }
        a.part_m[static_cast<int64_t>(item) * G + lane] = mv;
        a.part_l[static_cast<int64_t>(item) * G + lane] = lv;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(DB_O_FREE + (it & 1)));
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  griddep_launch_dependents();  // the combine may launch; it waits for this grid to end
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kDecTmemCols);
  }
}

// out[token b, head h, :] = sum_c w_c O_c / sum_c w_c l_c with w_c = 2^(m_c - max m)
// over the items c of (b, h / G); zeros for a sequence without keys.  One
// warp per (sequence, query head), four elements of head_dim per lane.
template <typename T, int G>
__global__ void __launch_bounds__(256) decode_combine_kernel(const DecodeArgs a, void* out, int64_t out_st,
                                                             int64_t out_sh, int num_q_heads) {
  griddep_wait();  // the partials of the decode kernel
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= a.num_seqs * num_q_heads) return;
  const int b = w / num_q_heads, h = w - b * num_q_heads;
  const int q0 = load_index(a.cu_q, b, a.len_i64);
  if (load_index(a.cu_q, b + 1, a.len_i64) - q0 != 1) return;
  const int L = load_index(a.seqused, b, a.len_i64);
  const int chunks = L > 0 ? (L + a.chunk - 1) / a.chunk : 0;
  const int kvh = h / G, g = h - kvh * G;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, den = 0.f;
  if (chunks > 0) {
    // m and l of up to 32 chunks in one round of loads across the lanes, then
    // the O rows eight chunks at a time, so the loads overlap.
    const int first = a.item_base[b] + kvh * chunks;
    float mmax = -INFINITY;
    for (int c = lane; c < chunks; c += 32) mmax = fmaxf(mmax, a.part_m[static_cast<int64_t>(first + c) * G + g]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, off));
    for (int c = lane; c < chunks; c += 32) {
      const int64_t row = static_cast<int64_t>(first + c) * G + g;
      den += ex2_approx(a.part_m[row] - mmax) * a.part_l[row];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
    for (int c0 = 0; c0 < chunks; c0 += 8) {
      float4 o[8];
      float w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u;
        const int64_t row = static_cast<int64_t>(first + min(c, chunks - 1)) * G + g;
        o[u] = reinterpret_cast<const float4*>(a.part_o + row * 128)[lane];
        w[u] = c < chunks ? ex2_approx(a.part_m[row] - mmax) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc[0] += w[u] * o[u].x;
        acc[1] += w[u] * o[u].y;
        acc[2] += w[u] * o[u].z;
        acc[3] += w[u] * o[u].w;
      }
    }
  }
  const float inv = 1.f / fmaxf(den, 1e-20f);
  T* dst = static_cast<T*>(out) + static_cast<int64_t>(q0) * out_st + static_cast<int64_t>(h) * out_sh + 4 * lane;
  uint2 v;
  v.x = Pack2<T>::pack(acc[0] * inv, acc[1] * inv);
  v.y = Pack2<T>::pack(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(dst) = v;
}

}  // namespace b200
