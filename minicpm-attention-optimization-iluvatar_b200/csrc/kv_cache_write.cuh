// kv_cache_write.cuh -- paged KV-cache write in the "flash" layout
// [num_blocks, block_size, num_kv_heads, head_dim], with the quantised
// variants the service's cache update selects.
//
// Semantics of IluvatarAttentionImpl.do_kv_cache_update
// (integration/vllm-plugin-FL-split-kv.patch:815-858 of the reference
// project), which calls vLLM's triton_reshape_and_cache_flash and
// triton_reshape_and_cache_flash_per_token_head_quant
// (vllm/v1/attention/ops/triton_reshape_and_cache_flash.py, vLLM 0.22):
//   * a token with slot < 0 is padding and writes nothing; otherwise row
//     (slot / bs, slot % bs, h) of each cache receives head h of the token;
//   * plain caches receive the key / value bits unchanged;
//   * fp8 per-tensor caches receive fp8(x / scale): the quotient rounded to
//     nearest in fp32, then to fp8 with round-to-nearest-even, saturating at
//     the largest finite value (a `cvt.rn.satfinite` conversion);
//   * per-token-head caches: s = max(max_d |x| / QMAX, 1e-6),
//     q = clamp(x * (1 / s), QMIN, QMAX), stored as int8 (truncation toward
//     zero, QMAX 127, QMIN -128) or fp8 e4m3 (RNE, +-448); s is stored in the
//     float scale cache of the same (block, slot, head).
// Quotients here are correctly rounded; vLLM's Triton code uses Triton's
// default fp32 division, so a quotient within a couple of fp32 ulps of an fp8
// rounding boundary may land one fp8 step apart from it.  The per-tensor
// divisor is fixed for a launch, so x / s is computed from the correctly
// rounded reciprocal y = 1/s and two residual corrections
// q <- q + (x - s q) y (Markstein's method; exact residuals by FMA): after
// the first correction q is within one ulp of x / s, and the second then
// yields the correctly rounded quotient, away from overflow and underflow.
// The result takes the sign of the first estimate (a zero keeps its sign; a
// subnormal quotient is far below the smallest fp8 value either way), and a
// first estimate beyond 2^20 in magnitude, which saturates every fp8 format
// used here, or a NaN, is kept as it is.
//
// Bandwidth kernel over the flattened (token, 8-element chunk) items: each
// thread owns one chunk of K and the same chunk of V per round, grid-stride
// with the grid sized to the resident capacity, and the next round's chunks
// and slot are loaded before the current round is converted and stored.
// Consecutive lanes hold consecutive chunks, so a head's head_dim/8 chunks sit
// in one aligned lane group and the per-head absolute maximum is a shuffle
// reduction inside it.  Index arithmetic is 32-bit (items and slots below
// 2^31, checked on the host), with shifts for power-of-two divisors.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "split_combine.cuh"

namespace b200 {

constexpr int kKvWriteThreads = 256;

enum KvMode : int { kKvCopy = 0, kKvFp8Tensor = 1, kKvPerTokenHead = 2 };
enum KvCacheElem : int { kElemSame = 0, kElemE4M3 = 1, kElemE5M2 = 2, kElemI8 = 3 };

struct KvWriteArgs {
  const void* k;
  const void* v;
  void* kc;
  void* vc;
  const void* slot;
  const float* k_scale;
  const float* v_scale;
  float* ksc;
  float* vsc;
  int64_t k_st, k_sh, v_st, v_sh;
  int64_t kc_sb, kc_st, kc_sh;
  int64_t vc_sb, vc_st, vc_sh;
  int64_t ks_sb, ks_st, ks_sh;
  int64_t vs_sb, vs_st, vs_sh;
  int64_t num_slots;
  int num_tokens, hkv, head_dim, block_size, slot_i64;
  uint32_t total_items;  // num_tokens * hkv * head_dim / 8
  int n_shift;           // log2(hkv * head_dim / 8), or -1
  int bs_shift;          // log2(block_size), or -1
};

__device__ __forceinline__ int64_t kv_load_index(const void* p, int64_t i, int is_i64) {
  return is_i64 ? static_cast<const int64_t*>(p)[i] : static_cast<int64_t>(static_cast<const int*>(p)[i]);
}

// Eight input elements of a chunk, raw (16 bytes for 2-byte types, 32 for f32).
template <typename T>
struct Chunk8 {
  uint4 w[sizeof(T) == 4 ? 2 : 1];
};

template <typename T>
__device__ __forceinline__ Chunk8<T> load_chunk(const T* p) {
  Chunk8<T> c;
  c.w[0] = reinterpret_cast<const uint4*>(p)[0];
  if (sizeof(T) == 4) c.w[sizeof(T) == 4 ? 1 : 0] = reinterpret_cast<const uint4*>(p)[1];
  return c;
}

template <typename T>
__device__ __forceinline__ void store_chunk(T* p, const Chunk8<T>& c) {
  reinterpret_cast<uint4*>(p)[0] = c.w[0];
  if (sizeof(T) == 4) reinterpret_cast<uint4*>(p)[1] = c.w[sizeof(T) == 4 ? 1 : 0];
}

template <typename T>
__device__ __forceinline__ void chunk_to_f32(const Chunk8<T>& c, float (&v)[8]) {
  load8<T>(reinterpret_cast<const T*>(&c.w[0]), v);
}

// Two floats -> two fp8 bytes (first value in the low byte), RNE, saturating.
template <int ELEM>
__device__ __forceinline__ uint32_t fp8x2(float a, float b) {
  return static_cast<uint32_t>(
      __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, ELEM == kElemE5M2 ? __NV_E5M2 : __NV_E4M3));
}

// Eight floats -> eight 1-byte cache elements, stored as two 4-byte words
// (the per-token-head caches pad each head by 4 bytes, so 8-byte alignment
// is not guaranteed).
template <int ELEM>
__device__ __forceinline__ void store_q8(uint8_t* p, const float (&q)[8]) {
  uint32_t w[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if (ELEM == kElemI8) {
      uint32_t r = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        r |= (static_cast<uint32_t>(__float2int_rz(q[4 * j + i])) & 0xffu) << (8 * i);
      w[j] = r;
    } else {
      w[j] = fp8x2<ELEM>(q[4 * j], q[4 * j + 1]) | (fp8x2<ELEM>(q[4 * j + 2], q[4 * j + 3]) << 16);
    }
  }
  reinterpret_cast<uint32_t*>(p)[0] = w[0];
  reinterpret_cast<uint32_t*>(p)[1] = w[1];
}

// A divisor fixed for the launch: s, its correctly rounded reciprocal, and
// whether that reciprocal is finite (s not below 2^-126).
struct FixedDivisor {
  float s, inv;
  bool finite;
};

__device__ __forceinline__ FixedDivisor make_divisor(float s) {
  FixedDivisor d;
  d.s = s;
  d.inv = __frcp_rn(s);
  d.finite = fabsf(d.inv) <= 3.4028234663852886e38f;
  return d;
}

// x[i] / s rounded to nearest (see the header comment), on packed pairs.
__device__ __forceinline__ void div_fixed8(const float (&x)[8], const FixedDivisor& d, float (&q)[8]) {
  if (!d.finite) {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __fdiv_rn(x[i], d.s);
    return;
  }
  const uint64_t inv = f2_pack(d.inv, d.inv), neg_s = f2_pack(-d.s, -d.s);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint64_t xv = f2_pack(x[2 * j], x[2 * j + 1]);
    const uint64_t q0 = f2_mul(xv, inv);
    const uint64_t q1 = f2_fma(f2_fma(q0, neg_s, xv), inv, q0);
    const uint64_t q2 = f2_fma(f2_fma(q1, neg_s, xv), inv, q1);
    float a0, a1, b0, b1;
    f2_unpack(q0, a0, a1);
    f2_unpack(q2, b0, b1);
    q[2 * j] = fabsf(a0) <= 0x1p20f ? copysignf(b0, a0) : a0;
    q[2 * j + 1] = fabsf(a1) <= 0x1p20f ? copysignf(b1, a1) : a1;
  }
}

// One correctly rounded quotient, same method, for any finite first
// estimate (the per-token-head scale max|x| / QMAX is stored, not saturated).
__device__ __forceinline__ float div_fixed(float x, const FixedDivisor& d) {
  if (!d.finite) return __fdiv_rn(x, d.s);
  const float q0 = __fmul_rn(x, d.inv);
  float q = __fmaf_rn(__fmaf_rn(-q0, d.s, x), d.inv, q0);
  q = __fmaf_rn(__fmaf_rn(-q, d.s, x), d.inv, q);
  return fabsf(q0) <= 3.4028234663852886e38f ? copysignf(q, q0) : q0;
}

// fp8(x / scale) for eight values.
template <int ELEM>
__device__ __forceinline__ void store_fp8_scaled(uint8_t* p, const float (&x)[8], const FixedDivisor& d) {
  float q[8];
  div_fixed8(x, d, q);
  store_q8<ELEM>(p, q);
}

// Per-token-head quantisation of one chunk: group = the head_dim/8 lanes of
// one head (aligned, a power of two dividing 32).  Every lane of the warp
// calls this; inactive lanes pass zeros and store nothing.
template <int ELEM, int GROUP>
__device__ __forceinline__ void quant_chunk_per_head(const float (&x)[8], bool active, uint8_t* dst,
                                                     float* scale_dst) {
  constexpr float kQMax = ELEM == kElemI8 ? 127.0f : 448.0f;
  constexpr float kQMin = ELEM == kElemI8 ? -128.0f : -448.0f;
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
  for (int off = 1; off < GROUP; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  constexpr FixedDivisor kQ{kQMax, 1.0f / kQMax, true};  // 1 / QMAX rounded to nearest at compile time
  const float s = fmaxf(div_fixed(amax, kQ), 1e-6f);
  const float inv = __frcp_rn(s);
  if (!active) return;
  float q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = fminf(fmaxf(__fmul_rn(x[i], inv), kQMin), kQMax);
  store_q8<ELEM>(dst, q);
  if (scale_dst) *scale_dst = s;
}

// One round's work of a thread: chunk i of token `token`, K and V.
template <typename T>
struct KvItem {
  Chunk8<T> k, v;
  int64_t slot;
  uint32_t token, i;
  bool valid;
};

template <typename T, int CPR>
__device__ __forceinline__ void fetch_item(const KvWriteArgs& a, uint32_t n, uint32_t it, KvItem<T>& x) {
  x.valid = it < a.total_items;
  x.slot = -1;
  if (!x.valid) return;
  x.token = a.n_shift >= 0 ? it >> a.n_shift : it / n;
  x.i = it - x.token * n;
  const uint32_t h = x.i / CPR, d = 8 * (x.i % CPR);
  x.k = load_chunk(static_cast<const T*>(a.k) + x.token * a.k_st + h * a.k_sh + d);
  x.v = load_chunk(static_cast<const T*>(a.v) + x.token * a.v_st + h * a.v_sh + d);
  x.slot = kv_load_index(a.slot, x.token, a.slot_i64);
}

// CPR = head_dim / 8 chunks per head (8, 16 or 32): the lane group of one head.
template <typename T, int MODE, int ELEM, int CPR>
__global__ void __launch_bounds__(kKvWriteThreads) kv_cache_write_kernel(const KvWriteArgs a) {
  const uint32_t n = static_cast<uint32_t>(a.hkv) * CPR;  // chunks per token and tensor
  FixedDivisor ks{}, vs{};
  if (MODE == kKvFp8Tensor) {
    ks = make_divisor(*a.k_scale);
    vs = make_divisor(*a.v_scale);
  }
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t warp_base = blockIdx.x * blockDim.x + (threadIdx.x & ~31u);
  KvItem<T> cur, nxt;
  fetch_item<T, CPR>(a, n, warp_base + lane, cur);
  // The loop bound is the warp's first item: every lane runs the same rounds
  // (the per-head shuffles need the whole warp).
  for (uint32_t base = warp_base; base < a.total_items; base += stride) {
    const uint32_t next = base + stride;
    if (next < a.total_items) fetch_item<T, CPR>(a, n, next + lane, nxt);
    const bool in_range = cur.valid && cur.slot >= 0 && cur.slot < a.num_slots;
    if (cur.valid && cur.slot >= a.num_slots && cur.i == 0) record_device_error(B200_DEVERR_SLOT_RANGE);
    uint32_t blk = 0, off = 0;
    if (in_range) {
      const uint32_t s32 = static_cast<uint32_t>(cur.slot);
      blk = a.bs_shift >= 0 ? s32 >> a.bs_shift : s32 / static_cast<uint32_t>(a.block_size);
      off = s32 - blk * static_cast<uint32_t>(a.block_size);
    }
    const uint32_t h = cur.i / CPR, d = 8 * (cur.i % CPR);
    const int64_t kco = static_cast<int64_t>(blk) * a.kc_sb + static_cast<int64_t>(off) * a.kc_st + h * a.kc_sh + d;
    const int64_t vco = static_cast<int64_t>(blk) * a.vc_sb + static_cast<int64_t>(off) * a.vc_st + h * a.vc_sh + d;
    if (MODE == kKvCopy) {
      if (in_range) {
        store_chunk(static_cast<T*>(a.kc) + kco, cur.k);
        store_chunk(static_cast<T*>(a.vc) + vco, cur.v);
      }
    } else {
      float kf[8], vf[8];
      chunk_to_f32(cur.k, kf);
      chunk_to_f32(cur.v, vf);
      if (!in_range) {
#pragma unroll
        for (int j = 0; j < 8; ++j) kf[j] = vf[j] = 0.0f;
      }
      uint8_t* kdst = static_cast<uint8_t*>(a.kc) + kco;
      uint8_t* vdst = static_cast<uint8_t*>(a.vc) + vco;
      if (MODE == kKvFp8Tensor) {
        if (in_range) {
          store_fp8_scaled<ELEM>(kdst, kf, ks);
          store_fp8_scaled<ELEM>(vdst, vf, vs);
        }
      } else {
        const bool leader = d == 0;
        quant_chunk_per_head<ELEM, CPR>(
            kf, in_range, kdst,
            leader ? a.ksc + static_cast<int64_t>(blk) * a.ks_sb + static_cast<int64_t>(off) * a.ks_st + h * a.ks_sh
                   : nullptr);
        quant_chunk_per_head<ELEM, CPR>(
            vf, in_range, vdst,
            leader ? a.vsc + static_cast<int64_t>(blk) * a.vs_sb + static_cast<int64_t>(off) * a.vs_st + h * a.vs_sh
                   : nullptr);
      }
    }
    cur = nxt;
  }
}

}  // namespace b200
