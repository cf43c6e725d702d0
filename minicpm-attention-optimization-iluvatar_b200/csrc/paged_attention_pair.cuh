// paged_attention_pair.cuh -- the paged prefill attention on CTA pairs.
//
// Same semantics, masking, split handling and epilogue as paged_attn_fwd_kernel
// (paged_attention.cuh).  The difference is the UMMA: a cluster of two CTAs on
// two SMs issues tcgen05.mma.cta_group::2 with M = 256 (each CTA supplies 128
// rows of A and receives its 128 rows of D), and B is split along N between
// the pair.  For S = Q K^T the leader CTA (rank 0) holds tokens 0..63 of every
// K tile and the peer tokens 64..127; for O += P V the leader holds head-dim
// columns 0..63 of every V tile and the peer 64..127.  Each SM therefore
// fetches and stores half of every K/V tile (16 TMA boxes instead of 32) and
// its tensor core reads half of B from its own shared memory, which halves the
// shared-memory traffic of the K/V operands.  No load uses cluster multicast:
// each CTA loads its own half into its own shared memory and its copies
// complete on a local "landed" barrier; warp 2 of each CTA forwards every
// landed fill to the leader's "full" barrier, on which the UMMA issuer waits.
//
// Work unit = (sequence, KV head, 4 query tiles = 4P positions, split).  The
// leader holds query tiles 0 and 1, the peer tiles 2 and 3; UMMA "tile t" is
// the leader's tile t stacked on the peer's tile t.  Per CTA the warp roles,
// the 5-slot-equivalent ring (10 slots of 16 KB), TMEM map and register split
// are those of paged_attn_fwd_kernel; only the leader's warp 1 issues UMMAs,
// and the commits that signal S/O/slot release arrive in both CTAs.  Every
// cross-CTA wait is bounded like the others; both CTAs meet on the cluster
// barrier before TMEM is freed and either CTA exits.
#pragma once

#include "paged_attention.cuh"

namespace b200 {

constexpr int kPairTilesPerUnit = 4;
constexpr int kPairSlots = 10;
constexpr uint32_t kPairSlotBytes = 16384;                      // half of a K or V tile
constexpr uint32_t kSmPairQ = 0;                                // this CTA's Q0, Q1
constexpr uint32_t kSmPairKV = 65536;
constexpr uint32_t kSmPairBar = kSmPairKV + kPairSlots * kPairSlotBytes;
constexpr uint32_t kSmPairBytes = kSmPairBar + 512;
constexpr uint32_t kAttnPairSmemAlloc = kSmPairBytes + 1024;

enum : int {
  PBAR_Q_LAND = 0,                             // local: this CTA's Q copies landed
  PBAR_Q = 1,                                  // leader: both CTAs' Q landed (count 2)
  PBAR_KV_LAND = 2,                            // local: + slot, this CTA's half landed
  PBAR_KV_FULL = PBAR_KV_LAND + kPairSlots,    // leader: + slot, both halves landed (count 2)
  PBAR_KV_EMPTY = PBAR_KV_FULL + kPairSlots,   // both: + slot (multicast commit)
  PBAR_S_FULL = PBAR_KV_EMPTY + kPairSlots,    // both: + tile (multicast commit)
  PBAR_P_FULL = PBAR_S_FULL + 2,               // leader: + tile, 4 warps x 2 CTAs
  PBAR_O_DONE = PBAR_P_FULL + 2,               // both: + tile (multicast commit)
  PBAR_DRAIN = PBAR_O_DONE + 2,                // leader
  PBAR_COUNT = PBAR_DRAIN + 1
};
static_assert(PBAR_COUNT * 8 + 8 <= 512, "barrier area");

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kAttnThreads, 1)
    paged_attn_fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                               const __grid_constant__ CUtensorMap tm_v, const AttnKernelArgs a) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  const int cluster_id = static_cast<int>(blockIdx.x >> 1);
  griddep_wait();  // launched as a programmatic dependent of the schedule kernel
  if (cluster_id >= *a.unit_count) return;  // uniform across the pair

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmPairBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmPairBar + PBAR_COUNT * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmPairBar + PBAR_COUNT * 8 + 4);
  auto bar = [&](int i) { return smem_addr(&bars[i]); };

  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const bool leader = rank == 0;
  // The leader's copy of a barrier, as a shared::cluster address.
  auto lbar = [&](int i) { return mapa_shared(smem_addr(&bars[i]), 0); };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int P = a.pos_per_tile;

  const int4 unit = a.units[cluster_id];
  const int seq = unit.x, qunit = unit.y, kvh = unit.z, split = unit.w;
  const UnitGeom ug = unit_geometry(load_index(a.cu_q, seq, a.len_i64), load_index(a.cu_q, seq + 1, a.len_i64),
                                    load_index(a.seqused, seq, a.len_i64), qunit, split, kPairTilesPerUnit * P,
                                    a.num_splits);
  const int n_tiles = ug.n_tiles;
  const bool two = ug.pos0 + P < ug.q_len;          // UMMA tile 1 has rows (leader's tile 1 at pos0 + P)
  const int my_pos0 = ug.pos0 + static_cast<int>(rank) * 2 * P;  // this CTA's tile 0

  if (threadIdx.x == 0) {
    mbar_init(bar(PBAR_Q_LAND), 1);
    mbar_init(bar(PBAR_Q), 2);
    for (int s = 0; s < kPairSlots; ++s) {
      mbar_init(bar(PBAR_KV_LAND + s), 1);
      mbar_init(bar(PBAR_KV_FULL + s), 2);
      mbar_init(bar(PBAR_KV_EMPTY + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(PBAR_S_FULL + t), 1);
      mbar_init(bar(PBAR_P_FULL + t), 8);
      mbar_init(bar(PBAR_O_DONE + t), 1);
    }
    mbar_init(bar(PBAR_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Barriers initialised in both CTAs before either arrives on the other's.
  cluster_sync();
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(tmem_slot), kAttnTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both halves of the pair's TMEM allocated before any UMMA
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAttnProducerRegs));
    if (warp == 0 && n_tiles > 0) {
      // ---------------------------------------------------------- producer (whole warp)
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        const int head0 = kvh * a.group;
        const int t0 = ug.q_begin + my_pos0;
        mbar_arrive_expect_tx(bar(PBAR_Q_LAND), (two ? 2 : 1) * 32768);
        tma_load_3d(sbase + kSmPairQ, &tm_q, bar(PBAR_Q_LAND), 0, head0, t0);
        tma_load_3d(sbase + kSmPairQ + 16384, &tm_q, bar(PBAR_Q_LAND), 64, head0, t0);
        if (two) {
          tma_load_3d(sbase + kSmPairQ + 32768, &tm_q, bar(PBAR_Q_LAND), 0, head0, t0 + P);
          tma_load_3d(sbase + kSmPairQ + 49152, &tm_q, bar(PBAR_Q_LAND), 64, head0, t0 + P);
        }
      }
      const int64_t bt_row = static_cast<int64_t>(seq) * a.bt_stride;
      const int my_slice = lane & 7;
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
      int issued = 0;
      for (int idx = 0; idx < 2 * n_tiles; ++idx) {
        const int j = idx >> 1;
        const bool is_v = idx & 1;
        const int slot = idx % kPairSlots;
        const uint32_t ph = (idx / kPairSlots) & 1;
        if (!is_v && j > 0) {
          pg_cur = pg_nxt;
          of_cur = of_nxt;
          if (j + 1 < n_tiles) lookup(j + 1, pg_nxt, of_nxt);
        }
        // K: this CTA's four 16-token slices (rank * 4 ..), both head-dim halves;
        // V: all eight slices, this CTA's head-dim half.
        const int c = is_v ? (lane & 7) : static_cast<int>(rank) * 4 + ((lane >> 1) & 3);
        const int page = __shfl_sync(0xffffffffu, pg_cur, c);
        const int off = __shfl_sync(0xffffffffu, of_cur, c);
        int ok = 1;
        if (lane == 0) {
          ok = mbar_wait(bar(PBAR_KV_EMPTY + slot), ph ^ 1, abort_flag);
          if (ok) mbar_arrive_expect_tx(bar(PBAR_KV_LAND + slot), kPairSlotBytes);
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        if (lane < 8) {
          const uint32_t dst = sbase + kSmPairKV + slot * kPairSlotBytes;
          if (is_v) {
            tma_load_4d(dst + c * 2048, &tm_v, bar(PBAR_KV_LAND + slot), static_cast<int>(rank) * 64, off, kvh, page);
          } else {
            const int half = lane & 1;
            tma_load_4d(dst + half * 8192 + (c & 3) * 2048, &tm_k, bar(PBAR_KV_LAND + slot), half * 64, off, kvh,
                        page);
          }
        }
        ++issued;
      }
      // Tail: the release of every slot's last fill (a UMMA commit that
      // arrives in both CTAs after the copies landed and were consumed).
      if (lane == 0 && !*abort_flag) {
        for (int s = 0; s < kPairSlots && s < issued; ++s) {
          const int last_idx = s + kPairSlots * ((issued - 1 - s) / kPairSlots);
          mbar_wait_drain(bar(PBAR_KV_EMPTY + s), (last_idx / kPairSlots) & 1);
        }
      }
      if (lane == 0 && *abort_flag) {
        // Abort: let this CTA's issued copies land before it can exit.
        mbar_wait_drain(bar(PBAR_Q_LAND), 0);
        for (int s = 0; s < kPairSlots && s < issued; ++s) {
          const int last_idx = s + kPairSlots * ((issued - 1 - s) / kPairSlots);
          mbar_wait_drain(bar(PBAR_KV_LAND + s), (last_idx / kPairSlots) & 1);
        }
      }
    } else if (warp == 2 && lane == 0 && n_tiles > 0) {
      // ---------------------------------------------------------- forwarder
      // This CTA's copies landed (local barriers) -> one arrival on the
      // leader's full barriers, which count both CTAs.
      bool ok = mbar_wait(bar(PBAR_Q_LAND), 0, abort_flag);
      if (ok) mbar_arrive_cluster(lbar(PBAR_Q));
      for (int idx = 0; ok && idx < 2 * n_tiles; ++idx) {
        const int slot = idx % kPairSlots;
        if (!mbar_wait(bar(PBAR_KV_LAND + slot), (idx / kPairSlots) & 1, abort_flag)) break;
        mbar_arrive_cluster(lbar(PBAR_KV_FULL + slot));
      }
    } else if (warp == 1 && lane == 0 && leader && n_tiles > 0) {
      // ---------------------------------------------------------- UMMA issuer (leader)
      constexpr uint32_t idesc_qk = umma_idesc_f16(kBF16, 256, 128, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_f16(kBF16, 256, 128, false, true);
      auto issue_s = [&](int t, uint32_t kslot) {
        const uint32_t q = sbase + kSmPairQ + t * 32768;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t qoff = (kk >> 2) * 16384 + (kk & 3) * 32;  // Q: 128 rows per head-dim half
          const uint32_t koff = (kk >> 2) * 8192 + (kk & 3) * 32;   // K: 64 rows per head-dim half
          umma_ss_pair(tmem + t * 128, umma_desc_sw128(q + qoff, 16, 1024), umma_desc_sw128(kslot + koff, 16, 1024),
                       idesc_qk, kk > 0);
        }
        tc_commit_pair_mc(bar(PBAR_S_FULL + t), 3);
      };
      auto issue_pv = [&](int t, uint32_t vslot, bool acc) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          umma_ts_pair(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, umma_desc_sw128(vslot + kk * 2048, 16384, 1024),
                       idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
        tc_commit_pair_mc(bar(PBAR_O_DONE + t), 3);
      };
      auto slot_addr = [&](int idx) { return sbase + kSmPairKV + (idx % kPairSlots) * kPairSlotBytes; };
      auto wait_full = [&](int idx) {
        return mbar_wait_cluster(bar(PBAR_KV_FULL + idx % kPairSlots), (idx / kPairSlots) & 1, abort_flag);
      };

      bool ok = mbar_wait_cluster(bar(PBAR_Q), 0, abort_flag) && wait_full(0);
      if (ok) {
        tc_fence_after();
        issue_s(0, slot_addr(0));
        if (two) issue_s(1, slot_addr(0));
        tc_commit_pair_mc(bar(PBAR_KV_EMPTY + 0), 3);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int vidx = 2 * j + 1, kidx = 2 * j + 2;
        const bool more = j + 1 < n_tiles;
        if (!wait_full(vidx) || !mbar_wait_cluster(bar(PBAR_P_FULL + 0), j & 1, abort_flag)) break;
        tc_fence_after();
        issue_pv(0, slot_addr(vidx), j > 0);
        if (more) {
          if (!wait_full(kidx)) break;
          tc_fence_after();
          issue_s(0, slot_addr(kidx));
        }
        if (two) {
          if (!mbar_wait_cluster(bar(PBAR_P_FULL + 1), j & 1, abort_flag)) break;
          tc_fence_after();
          issue_pv(1, slot_addr(vidx), j > 0);
          if (more) issue_s(1, slot_addr(kidx));
        }
        tc_commit_pair_mc(bar(PBAR_KV_EMPTY + vidx % kPairSlots), 3);
        if (more) tc_commit_pair_mc(bar(PBAR_KV_EMPTY + kidx % kPairSlots), 3);
      }
      tc_commit_pair(bar(PBAR_DRAIN));
      mbar_wait_drain(bar(PBAR_DRAIN), 0);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kAttnSoftmaxRegs));
    // ------------------------------------------------------------ softmax (tile t of this CTA)
    const int t = (warp - 4) >> 2;
    if (t == 0 || two) {
      const int quarter = warp & 3;
      const int row = quarter * 32 + lane;
      const int tile_pos0 = my_pos0 + t * P;
      const int row_pos = tile_pos0 + row / a.group;
      const int row_head = kvh * a.group + row % a.group;
      const bool row_valid = row_pos < ug.q_len;
      const int q_abs_first = ug.q_abs_min + (tile_pos0 - ug.pos0);  // this tile's first row
      const int q_abs = q_abs_first + row / a.group;
      const int row_hi = min(ug.split_end, q_abs + 1);
      const int unmasked_hi = min(ug.split_end, q_abs_first + 1);
      const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
      const uint32_t s_addr = tmem + lane_base + t * 128;
      const uint32_t o_addr = tmem + lane_base + 256 + t * 128;
      const float sl2 = a.scale_log2;
      const uint32_t p_full_leader = lbar(PBAR_P_FULL + t);
      const int last_start = ug.kv_lo + (n_tiles - 1) * kAttnTileN;
      const int v_tail_from = max(ug.seq_len - last_start, 0);
      const int v_tail_to = min(((ug.kv_hi + kAttnSlice - 1) / kAttnSlice) * kAttnSlice - last_start, kAttnTileN);

      float m_used = -INFINITY;
      float l = 0.f;
      bool aborted = false;
      for (int j = 0; j < n_tiles; ++j) {
        if (!mbar_wait(bar(PBAR_S_FULL + t), j & 1, abort_flag)) {
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
            for (int c = 0; c < 32; ++c) {
              const int col = c4 * 32 + c;
              if (col < lo || col >= hi) sr[c4][c] = __float_as_uint(-INFINITY);
            }
        }
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
          for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              mx[k] = fmax3(mx[k], __uint_as_float(sr[c4][16 * h + 2 * k]), __uint_as_float(sr[c4][16 * h + 2 * k + 1]));
        const float mxa = fmax3(mx[0], mx[1], mx[2]), mxb = fmax3(mx[3], mx[4], mx[5]);
        const float m_cand = fmaxf(m_used, fmax3(mxa, mxb, fmaxf(mx[6], mx[7])) * sl2);
        const bool raise = m_cand > m_used + kRescaleThreshold;
        if (__any_sync(0xffffffffu, raise)) {
          const float alpha = raise ? ex2_approx(m_used - m_cand) : 1.f;
          if (j > 0) {
            if (!mbar_wait(bar(PBAR_O_DONE + t), (j - 1) & 1, abort_flag)) {
              aborted = true;
              break;
            }
            tc_fence_after();
#pragma unroll 1
            for (int c8 = 0; c8 < 8; ++c8) {
              uint32_t o[16];
              tmem_ld16(o_addr + 16 * c8, o);
              tmem_wait_ld16(o);
#pragma unroll
              for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              tmem_st16(o_addr + 16 * c8, o);
            }
          }
          if (raise) {
            l *= alpha;
            m_used = m_cand;
          }
        }
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        const uint64_t sl2_2 = f2_pack(sl2, sl2), negm_2 = f2_pack(neg_m, neg_m);
        uint64_t sum_a = f2_pack(0.f, 0.f), sum_b = sum_a;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
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
        {
          float a0, a1;
          f2_unpack(f2_add(sum_a, sum_b), a0, a1);
          l += a0 + a1;
        }
        if (t == 0 && j == n_tiles - 1 && v_tail_from < v_tail_to) {
          // Zero this CTA's half of the V rows past the sequence end (NaN-safe
          // PV, as the reference's masked V load), once its copy has landed.
          const int vidx = 2 * j + 1;
          if (!mbar_wait(bar(PBAR_KV_LAND + vidx % kPairSlots), (vidx / kPairSlots) & 1, abort_flag)) {
            aborted = true;
            break;
          }
          const uint32_t vbase = sbase + kSmPairKV + (vidx % kPairSlots) * kPairSlotBytes;
          const int n16 = (v_tail_to - v_tail_from) * 8;  // 16-byte pieces of this CTA's 128-byte rows
          for (int i = threadIdx.x - 128; i < n16; i += 128) {
            const int r = v_tail_from + (i >> 3);
            st_shared_v4(vbase + r * 128 + (i & 7) * 16, 0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(p_full_leader);  // one arrival per softmax warp per CTA
      }

      if (!aborted && n_tiles > 0) {
        if (!mbar_wait(bar(PBAR_O_DONE + t), (n_tiles - 1) & 1, abort_flag)) aborted = true;
        tc_fence_after();
      }
      if (!aborted) {
        const float inv = 1.f / fmaxf(l, 1e-20f);
        const int tok = ug.q_begin + row_pos;
        T* dst;
        if (a.num_splits == 1) {
          dst = static_cast<T*>(a.out) + static_cast<int64_t>(tok) * a.out_st + static_cast<int64_t>(row_head) * a.out_sh;
        } else {
          const int64_t rowi = (static_cast<int64_t>(split) * a.total_q + tok) * a.num_q_heads + row_head;
          dst = static_cast<T*>(a.o_split) + rowi * kAttnHeadDim;
          if (row_valid) {
            a.m_split[rowi] = (l > 0.f) ? m_used * 0.69314718055994530942f : -INFINITY;
            a.l_split[rowi] = l;
          }
        }
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
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no remote arrival or UMMA may target a CTA that has left
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kAttnTmemCols);
  }
}

}  // namespace b200
