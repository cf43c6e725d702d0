// paged_attention.cuh -- causal varlen paged prefill attention for sm_100a.
//
// Semantics follow the reference Split-KV kernel
// (kernels/triton_split_kv_paged.py:63-155 of the reference project):
//   * query row i of sequence b sits at absolute position L_b - q_len_b + i;
//   * split s of S covers keys [s * ceil(L/S), min((s + 1) * ceil(L/S), L));
//   * a key is valid for a row iff it is inside the split and <= the row's
//     absolute position; a row with no valid key keeps m = -inf, l = 0, O = 0;
//   * S == 1 writes the normalised output directly; S > 1 writes the
//     normalised partial O (in the query dtype) plus m (natural-log units)
//     and l, which b200_split_combine reduces.
//
// Work unit = (sequence, KV head, query tile, split).  A query tile packs
// the G = Hq / KH query heads that share one KV head with 128 / G query
// positions into the 128 rows of one UMMA M dimension (row r = position
// r / G, head r % G), so every K/V tile fetched from HBM feeds all G heads.
//
// One CTA per unit, 6 warps:
//   warp 0      TMA producer: Q once, then K and V tiles of 128 tokens as
//               8 page slices of 16 tokens x 2 half-rows each, addressed
//               through the block table (per-page TMA gather).  Slices past
//               the unit's last key load from an out-of-range page index, so
//               TMA fills zeros and never touches memory outside the cache.
//   warp 1      TMEM owner and single-thread UMMA issuer:
//               S[j%2] = Q K_j^T (M128 N128 K128), O += P_{j-1} V_{j-1}.
//   warps 2..5  softmax warpgroup, one query row per thread: reads S from
//               TMEM, masks, online softmax in base 2, rescales O in TMEM,
//               writes P (bf16/f16) to shared memory, final normalise+store.
// TMEM: S double buffer at columns [0,128) and [128,256), O at [256,384).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "sm100_ptx.cuh"

namespace b200 {

constexpr int kAttnTileM = 128;   // rows per query tile
constexpr int kAttnTileN = 128;   // KV tokens per tile
constexpr int kAttnHeadDim = 128; // head_dim handled by this kernel
constexpr int kAttnSlice = 16;    // KV tokens per TMA box (page slice)
constexpr int kAttnThreads = 192;
constexpr int kAttnTmemCols = 512;
constexpr int kColS0 = 0, kColS1 = 128, kColO = 256;

// Shared memory map (offsets from a 1024-aligned base).
constexpr uint32_t kSmQ = 0;                       // 2 x 16 KB (d halves)
constexpr uint32_t kSmK = 32768;                   // 2 stages x 2 halves x 16 KB
constexpr uint32_t kSmV = kSmK + 65536;            // 2 stages x 2 halves x 16 KB
constexpr uint32_t kSmP = kSmV + 65536;            // 2 x 16 KB (kv halves)
constexpr uint32_t kSmBar = kSmP + 32768;          // mbarriers
constexpr uint32_t kSmBytes = kSmBar + 256;
constexpr uint32_t kAttnSmemAlloc = kSmBytes + 1024;  // + alignment slack

// mbarrier slots
enum : int {
  BAR_Q = 0,
  BAR_K_FULL = 1,   // +stage
  BAR_K_EMPTY = 3,  // +stage
  BAR_V_FULL = 5,   // +stage
  BAR_V_EMPTY = 7,  // +stage
  BAR_S_FULL = 9,   // +stage
  BAR_S_FREE = 11,  // +stage
  BAR_P_FULL = 13,
  BAR_O_DONE = 14,
  BAR_DRAIN = 15,
  BAR_COUNT = 16
};

struct AttnKernelArgs {
  const void* block_table;
  const void* cu_q;
  const void* seqused;
  void* out;
  void* o_split;
  float* m_split;
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
  int group;          // G = Hq / KH
  int pos_per_tile;   // 128 / G
  int block_size;
  int num_blocks;
  int num_splits;
  float scale_log2;   // softmax_scale * log2(e)
};

__device__ __forceinline__ int load_index(const void* p, int64_t i, int is_i64) {
  return is_i64 ? static_cast<int>(static_cast<const int64_t*>(p)[i]) : static_cast<const int*>(p)[i];
}

// Geometry of one work unit; shared by the scheduler (cost) and the kernel.
struct UnitGeom {
  int q_begin, q_len, seq_len;
  int pos0, split_begin, split_end;
  int kv_lo, kv_hi, n_tiles;
  int q_abs_min;
};

__device__ __forceinline__ UnitGeom unit_geometry(int q_begin, int q_end, int seq_len, int qtile, int split,
                                                  int pos_per_tile, int num_splits) {
  UnitGeom u;
  u.q_begin = q_begin;
  u.q_len = q_end - q_begin;
  u.seq_len = seq_len;
  u.pos0 = qtile * pos_per_tile;
  const int rows = min(pos_per_tile, u.q_len - u.pos0);
  u.q_abs_min = seq_len - u.q_len + u.pos0;
  const int q_abs_max = u.q_abs_min + rows - 1;
  const int L = max(seq_len, 0);
  const int split_size = (L + num_splits - 1) / num_splits;
  u.split_begin = split * split_size;
  u.split_end = min(u.split_begin + split_size, L);
  u.kv_hi = min(u.split_end, q_abs_max + 1);
  u.kv_lo = (u.split_begin / kAttnSlice) * kAttnSlice;
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

// Wait without the abort short-cut: used on the abort path to let copies
// and MMAs already in flight land before the CTA exits.
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > B200_WAIT_LIMIT_NS) {
      record_device_error(B200_DEVERR_WAIT_TIMEOUT);
      return;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads, 1)
    paged_attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const AttnKernelArgs a) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  if (static_cast<int>(blockIdx.x) >= *a.unit_count) return;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmBar + BAR_COUNT * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmBar + BAR_COUNT * 8 + 4);
  auto bar = [&](int i) { return smem_addr(&bars[i]); };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  const int4 unit = a.units[blockIdx.x];
  const int seq = unit.x, qtile = unit.y, kvh = unit.z, split = unit.w;
  const UnitGeom ug = unit_geometry(load_index(a.cu_q, seq, a.len_i64), load_index(a.cu_q, seq + 1, a.len_i64),
                                    load_index(a.seqused, seq, a.len_i64), qtile, split, a.pos_per_tile,
                                    a.num_splits);
  const int n_tiles = ug.n_tiles;

  if (threadIdx.x == 0) {
    mbar_init(bar(BAR_Q), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(BAR_K_FULL + s), 1);
      mbar_init(bar(BAR_K_EMPTY + s), 1);
      mbar_init(bar(BAR_V_FULL + s), 1);
      mbar_init(bar(BAR_V_EMPTY + s), 1);
      mbar_init(bar(BAR_S_FULL + s), 1);
      mbar_init(bar(BAR_S_FREE + s), 4);
    }
    mbar_init(bar(BAR_P_FULL), 4);
    mbar_init(bar(BAR_O_DONE), 1);
    mbar_init(bar(BAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int head0 = kvh * a.group;
      const int t0 = ug.q_begin + ug.pos0;
      mbar_arrive_expect_tx(bar(BAR_Q), 2 * 16384);
      tma_load_3d(sbase + kSmQ, &tm_q, bar(BAR_Q), 0, head0, t0);
      tma_load_3d(sbase + kSmQ + 16384, &tm_q, bar(BAR_Q), 64, head0, t0);
      int kfills[2] = {0, 0}, vfills[2] = {0, 0};
      const int64_t bt_row = static_cast<int64_t>(seq) * a.bt_stride;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int tile_start = ug.kv_lo + j * kAttnTileN;
        int page[8], off[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int pos = tile_start + c * kAttnSlice;
          page[c] = a.num_blocks;  // out of range: TMA fills zeros
          off[c] = 0;
          if (pos < ug.kv_hi) {
            const int lp = pos / a.block_size;
            off[c] = pos - lp * a.block_size;
            if (lp < a.bt_cols) page[c] = load_index(a.block_table, bt_row + lp, a.bt_i64);
          }
        }
        if (!mbar_wait(bar(BAR_K_EMPTY + st), ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(bar(BAR_K_FULL + st), 2 * 16384);
        const uint32_t kdst = sbase + kSmK + st * 32768;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          tma_load_4d(kdst + c * 2048, &tm_k, bar(BAR_K_FULL + st), 0, off[c], kvh, page[c]);
          tma_load_4d(kdst + 16384 + c * 2048, &tm_k, bar(BAR_K_FULL + st), 64, off[c], kvh, page[c]);
        }
        ++kfills[st];
        if (!mbar_wait(bar(BAR_V_EMPTY + st), ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(bar(BAR_V_FULL + st), 2 * 16384);
        const uint32_t vdst = sbase + kSmV + st * 32768;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          tma_load_4d(vdst + c * 2048, &tm_v, bar(BAR_V_FULL + st), 0, off[c], kvh, page[c]);
          tma_load_4d(vdst + 16384 + c * 2048, &tm_v, bar(BAR_V_FULL + st), 64, off[c], kvh, page[c]);
        }
        ++vfills[st];
      }
      if (*abort_flag) {
        // Let every issued copy land before the CTA can exit.
        mbar_wait_drain(bar(BAR_Q), 0);
        for (int st = 0; st < 2; ++st) {
          if (kfills[st] > 0) mbar_wait_drain(bar(BAR_K_FULL + st), (kfills[st] - 1) & 1);
          if (vfills[st] > 0) mbar_wait_drain(bar(BAR_V_FULL + st), (vfills[st] - 1) & 1);
        }
      } else {
        // Producer tail: the UMMA commits that release the last K and V stages
        // must have arrived before this CTA's shared memory can be reused.
        for (int st = 0; st < 2; ++st) {
          if (kfills[st] > 0) mbar_wait_drain(bar(BAR_K_EMPTY + st), (kfills[st] - 1) & 1);
          if (vfills[st] > 0) mbar_wait_drain(bar(BAR_V_EMPTY + st), (vfills[st] - 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = umma_idesc_f16(kBF16, 128, 128, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_f16(kBF16, 128, 128, false, true);
      bool ok = mbar_wait(bar(BAR_Q), 0, abort_flag);
      for (int j = 0; ok && j <= n_tiles; ++j) {
        if (j < n_tiles) {
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(bar(BAR_K_FULL + st), ph, abort_flag)) break;
          if (!mbar_wait(bar(BAR_S_FREE + st), ph ^ 1, abort_flag)) break;
          tc_fence_after();
          const uint32_t d_s = tmem + (st ? kColS1 : kColS0);
          const uint32_t kbase = sbase + kSmK + st * 32768;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_ss(d_s, umma_desc_sw128(sbase + kSmQ + koff, 16, 1024), umma_desc_sw128(kbase + koff, 16, 1024),
                    idesc_qk, kk > 0);
          }
          tc_commit(bar(BAR_S_FULL + st));
          tc_commit(bar(BAR_K_EMPTY + st));
        }
        if (j > 0) {
          const int i = j - 1;
          const int st = i & 1;
          const uint32_t ph = (i >> 1) & 1;
          if (!mbar_wait(bar(BAR_V_FULL + st), ph, abort_flag)) break;
          if (!mbar_wait(bar(BAR_P_FULL), i & 1, abort_flag)) break;
          tc_fence_after();
          const uint32_t vbase = sbase + kSmV + st * 32768;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t poff = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_ss(tmem + kColO, umma_desc_sw128(sbase + kSmP + poff, 16, 1024),
                    umma_desc_sw128(vbase + kk * 2048, 16384, 1024), idesc_pv, (i > 0 || kk > 0));
          }
          tc_commit(bar(BAR_O_DONE));
          tc_commit(bar(BAR_V_EMPTY + st));
        }
      }
      if (*abort_flag) {
        tc_commit(bar(BAR_DRAIN));
        mbar_wait_drain(bar(BAR_DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int row = quarter * 32 + lane;
    const int row_pos = ug.pos0 + row / a.group;
    const int row_head = kvh * a.group + row % a.group;
    const bool row_valid = row_pos < ug.q_len;
    const int q_abs = ug.q_abs_min + row / a.group;
    const int row_hi = min(ug.split_end, q_abs + 1);
    const int tiles_unmasked_hi = min(ug.split_end, ug.q_abs_min + 1);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = a.scale_log2;
    // V rows [v_tail_from, v_tail_to) of the last tile: loaded page rows at or past L.
    const int last_start = ug.kv_lo + (n_tiles - 1) * kAttnTileN;
    const int v_tail_from = max(ug.seq_len - last_start, 0);
    const int v_tail_to = min(((ug.kv_hi + kAttnSlice - 1) / kAttnSlice) * kAttnSlice - last_start, kAttnTileN);

    float m2 = -INFINITY;
    float l = 0.f;
    bool aborted = false;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!mbar_wait(bar(BAR_S_FULL + st), ph, abort_flag)) {
        aborted = true;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t sr[4][32];
      const uint32_t s_addr = tmem + lane_base + (st ? kColS1 : kColS0);
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(s_addr + 32 * c4, sr[c4]);
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) tmem_wait_ld(sr[c4]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_S_FREE + st));

      const int tile_start = ug.kv_lo + j * kAttnTileN;
      const bool need_mask = (tile_start < ug.split_begin) || (tile_start + kAttnTileN > tiles_unmasked_hi);
      if (need_mask) {
        const int lo = ug.split_begin - tile_start;
        const int hi = row_hi - tile_start;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int col = c4 * 32 + c;
            if (col < lo || col >= hi) sr[c4][c] = __float_as_uint(-INFINITY);
          }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        mx0 = fmaxf(mx0, __uint_as_float(sr[0][c]));
        mx1 = fmaxf(mx1, __uint_as_float(sr[1][c]));
        mx2 = fmaxf(mx2, __uint_as_float(sr[2][c]));
        mx3 = fmaxf(mx3, __uint_as_float(sr[3][c]));
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      const float m_new = fmaxf(m2, mx * sl2);
      const float safe = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2_approx(m2 - safe);
      const float neg_safe = -safe;

      uint32_t pk[64];
      float sum0 = 0.f, sum1 = 0.f, sum2 = 0.f, sum3 = 0.f;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c4][c]), sl2, neg_safe));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sr[c4][c + 1]), sl2, neg_safe));
          if (c & 2) {
            sum2 += p0;
            sum3 += p1;
          } else {
            sum0 += p0;
            sum1 += p1;
          }
          pk[c4 * 16 + c / 2] = Pack2<T>::pack(p0, p1);
        }
      }
      l = l * alpha + ((sum0 + sum1) + (sum2 + sum3));
      m2 = m_new;

      if (j > 0) {
        // PV of the previous tile must be done before O is rescaled and P is overwritten.
        if (!mbar_wait(bar(BAR_O_DONE), (j - 1) & 1, abort_flag)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          const uint32_t o_addr = tmem + lane_base + kColO;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t o[32];
            tmem_ld32(o_addr + 32 * c4, o);
            tmem_wait_ld(o);
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(o_addr + 32 * c4, o);
          }
          tmem_wait_st();
        }
      }
      // P row -> shared memory, K-major with the 128-byte swizzle (16-byte chunk c of
      // row r lands at chunk c ^ (r % 8)).
      const uint32_t p_row = sbase + kSmP + row * 128;
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        const uint32_t addr = p_row + (ch >> 3) * 16384 + (((ch & 7) ^ (row & 7)) << 4);
        st_shared_v4(addr, pk[ch * 4 + 0], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
      }
      if (j == n_tiles - 1 && v_tail_from < v_tail_to) {
        // Rows of the last page past the sequence end may hold anything (NaN
        // included); P is 0 there but 0 * NaN is NaN, so zero those V rows,
        // as the reference's masked V load does (triton_split_kv_paged.py:122).
        if (!mbar_wait(bar(BAR_V_FULL + st), ph, abort_flag)) {
          aborted = true;
          break;
        }
        const uint32_t vbase = sbase + kSmV + st * 32768;
        const int n16 = (v_tail_to - v_tail_from) * 16;  // 16-byte pieces over both halves
        for (int i = threadIdx.x - 64; i < n16; i += 128) {
          const int r = v_tail_from + (i >> 4);
          const int half = (i >> 3) & 1;
          st_shared_v4(vbase + half * 16384 + r * 128 + (i & 7) * 16, 0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_P_FULL));  // one arrival per softmax warp
    }

    // ------------------------------------------------------------ epilogue
    if (!aborted && n_tiles > 0) {
      if (!mbar_wait(bar(BAR_O_DONE), (n_tiles - 1) & 1, abort_flag)) aborted = true;
      tc_fence_after();
    }
    if (!aborted) {
      const float inv = 1.f / fmaxf(l, 1e-20f);
      const int t = ug.q_begin + row_pos;
      T* dst;
      if (a.num_splits == 1) {
        dst = static_cast<T*>(a.out) + static_cast<int64_t>(t) * a.out_st + static_cast<int64_t>(row_head) * a.out_sh;
      } else {
        const int64_t rowi = (static_cast<int64_t>(split) * a.total_q + t) * a.num_q_heads + row_head;
        dst = static_cast<T*>(a.o_split) + rowi * kAttnHeadDim;
        if (row_valid) {
          a.m_split[rowi] = (m2 == -INFINITY) ? -INFINITY : m2 * 0.69314718055994530942f;
          a.l_split[rowi] = l;
        }
      }
      const uint32_t o_addr = tmem + lane_base + kColO;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[32];
        if (n_tiles > 0) {
          tmem_ld32(o_addr + 32 * c4, o);
          tmem_wait_ld(o);
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
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
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Device-side work list: one block, bucket sort of units by KV-tile count,
// heaviest first, so the hardware's in-order CTA dispatch approximates a
// longest-processing-time schedule.  No host synchronisation is needed: the
// attention grid is sized to an upper bound and surplus CTAs exit at once.
// ---------------------------------------------------------------------------
constexpr int kSchedThreads = 1024;
constexpr int kSchedBuckets = 2048;

struct SchedArgs {
  const void* cu_q;
  const void* seqused;
  int len_i64;
  int num_seqs;
  int pos_per_tile;
  int num_kv_heads;
  int num_splits;
  int capacity;
  int* tile_base;  // [num_seqs + 1]
  int4* units;
  int* unit_count;
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

__global__ void __launch_bounds__(kSchedThreads, 1) attn_schedule_kernel(const SchedArgs a) {
  __shared__ int hist[kSchedBuckets];
  __shared__ int warp_sums[32];
  __shared__ int s_total_tiles;

  // 1. query tiles per sequence, exclusive prefix over sequences.
  int carry = 0;
  for (int base = 0; base < a.num_seqs; base += kSchedThreads) {
    const int b = base + threadIdx.x;
    int n = 0;
    if (b < a.num_seqs) {
      const int ql = load_index(a.cu_q, b + 1, a.len_i64) - load_index(a.cu_q, b, a.len_i64);
      n = ql > 0 ? (ql + a.pos_per_tile - 1) / a.pos_per_tile : 0;
    }
    int total;
    const int before = block_exclusive_scan(n, warp_sums, total);
    if (b < a.num_seqs) a.tile_base[b] = carry + before;
    carry += total;
  }
  if (threadIdx.x == 0) {
    a.tile_base[a.num_seqs] = carry;
    s_total_tiles = carry;
  }
  for (int i = threadIdx.x; i < kSchedBuckets; i += kSchedThreads) hist[i] = 0;
  __syncthreads();

  const int per_tile = a.num_kv_heads * a.num_splits;
  const int total_units = min(s_total_tiles * per_tile, a.capacity);

  auto decode = [&](int u, int& seq, int& qtile, int& kvh, int& split, int& bucket) {
    const int tile = u / per_tile;
    const int rem = u - tile * per_tile;
    kvh = rem / a.num_splits;
    split = rem - kvh * a.num_splits;
    int lo = 0, hi = a.num_seqs - 1;  // last seq with tile_base[seq] <= tile
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.tile_base[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    qtile = tile - a.tile_base[seq];
    const UnitGeom g = unit_geometry(load_index(a.cu_q, seq, a.len_i64), load_index(a.cu_q, seq + 1, a.len_i64),
                                     load_index(a.seqused, seq, a.len_i64), qtile, split, a.pos_per_tile,
                                     a.num_splits);
    bucket = min(g.n_tiles, kSchedBuckets - 1);
  };

  // 2. histogram of KV-tile counts.
  for (int u = threadIdx.x; u < total_units; u += kSchedThreads) {
    int seq, qtile, kvh, split, bucket;
    decode(u, seq, qtile, kvh, split, bucket);
    atomicAdd(&hist[bucket], 1);
  }
  __syncthreads();
  // 3. bucket offsets, heaviest bucket first.
  {
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
  __syncthreads();
  // 4. scatter.
  for (int u = threadIdx.x; u < total_units; u += kSchedThreads) {
    int seq, qtile, kvh, split, bucket;
    decode(u, seq, qtile, kvh, split, bucket);
    const int slot = atomicAdd(&hist[bucket], 1);
    a.units[slot] = make_int4(seq, qtile, kvh, split);
  }
  if (threadIdx.x == 0) *a.unit_count = total_units;
}

}  // namespace b200
