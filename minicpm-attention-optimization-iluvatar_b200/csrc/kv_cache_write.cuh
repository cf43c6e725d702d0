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
// Divisions here are correctly rounded (div.rn); vLLM's Triton code uses
// Triton's default fp32 division, so a quotient within a couple of fp32 ulps
// of an fp8 rounding boundary may land one fp8 step apart from it.
//
// Bandwidth kernel: one warp per token (grid-stride over tokens, grid sized to
// the resident capacity), lane i of a round owns the 8-element chunk i of the
// token's [num_kv_heads * head_dim] row; with head_dim/8 lanes per head the
// per-head absolute maximum is a shuffle reduction inside an aligned lane group.
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

// fp8(x / scale) for eight values.
template <int ELEM>
__device__ __forceinline__ void store_fp8_scaled(uint8_t* p, const float (&x)[8], float scale) {
  float q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = __fdiv_rn(x[i], scale);
  store_q8<ELEM>(p, q);
}

// Per-token-head quantisation of one chunk: group = the head_dim/8 lanes of
// one head (aligned, a power of two dividing 32).  Every lane of the warp
// calls this; inactive lanes pass zeros and store nothing.
template <int ELEM>
__device__ __forceinline__ void quant_chunk_per_head(const float (&x)[8], int group, bool active, uint8_t* dst,
                                                     float* scale_dst) {
  constexpr float kQMax = ELEM == kElemI8 ? 127.0f : 448.0f;
  constexpr float kQMin = ELEM == kElemI8 ? -128.0f : -448.0f;
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[i]));
  for (int off = 1; off < group; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float s = fmaxf(__fdiv_rn(amax, kQMax), 1e-6f);
  const float inv = __fdiv_rn(1.0f, s);
  if (!active) return;
  float q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = fminf(fmaxf(__fmul_rn(x[i], inv), kQMin), kQMax);
  store_q8<ELEM>(dst, q);
  if (scale_dst) *scale_dst = s;
}

template <typename T, int MODE, int ELEM>
__global__ void __launch_bounds__(kKvWriteThreads) kv_cache_write_kernel(const KvWriteArgs a) {
  const int lane = threadIdx.x & 31;
  const int cpr = a.head_dim >> 3;  // chunks per head: 8, 16 or 32
  const int n = a.hkv * cpr;        // chunks per token and tensor
  float ks = 1.0f, vs = 1.0f;
  if (MODE == kKvFp8Tensor) {
    ks = *a.k_scale;
    vs = *a.v_scale;
  }
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  int64_t token = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  int64_t slot_n = token < a.num_tokens ? kv_load_index(a.slot, token, a.slot_i64) : -1;
  for (; token < a.num_tokens; token += nwarps) {
    const int64_t slot = slot_n;
    if (token + nwarps < a.num_tokens) slot_n = kv_load_index(a.slot, token + nwarps, a.slot_i64);
    if (slot < 0) continue;
    if (slot >= a.num_slots) {
      if (lane == 0) record_device_error(B200_DEVERR_SLOT_RANGE);
      continue;
    }
    const int64_t blk = slot / a.block_size, off = slot - blk * a.block_size;
    const T* ktok = static_cast<const T*>(a.k) + token * a.k_st;
    const T* vtok = static_cast<const T*>(a.v) + token * a.v_st;
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const bool active = i < n;
      const int h = i / cpr, d = 8 * (i - h * cpr);
      Chunk8<T> kx{}, vx{};
      if (active) {
        kx = load_chunk(ktok + h * a.k_sh + d);
        vx = load_chunk(vtok + h * a.v_sh + d);
      }
      if (MODE == kKvCopy) {
        if (active) {
          store_chunk(static_cast<T*>(a.kc) + blk * a.kc_sb + off * a.kc_st + h * a.kc_sh + d, kx);
          store_chunk(static_cast<T*>(a.vc) + blk * a.vc_sb + off * a.vc_st + h * a.vc_sh + d, vx);
        }
        continue;
      }
      uint8_t* kdst = static_cast<uint8_t*>(a.kc) + blk * a.kc_sb + off * a.kc_st + h * a.kc_sh + d;
      uint8_t* vdst = static_cast<uint8_t*>(a.vc) + blk * a.vc_sb + off * a.vc_st + h * a.vc_sh + d;
      float kf[8], vf[8];
      if (active) {
        chunk_to_f32(kx, kf);
        chunk_to_f32(vx, vf);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) kf[j] = vf[j] = 0.0f;
      }
      if (MODE == kKvFp8Tensor) {
        if (active) {
          store_fp8_scaled<ELEM>(kdst, kf, ks);
          store_fp8_scaled<ELEM>(vdst, vf, vs);
        }
      } else {
        const bool leader = d == 0;
        quant_chunk_per_head<ELEM>(kf, cpr, active, kdst,
                                   leader ? a.ksc + blk * a.ks_sb + off * a.ks_st + h * a.ks_sh : nullptr);
        quant_chunk_per_head<ELEM>(vf, cpr, active, vdst,
                                   leader ? a.vsc + blk * a.vs_sb + off * a.vs_st + h * a.vs_sh : nullptr);
      }
    }
  }
}

}  // namespace b200
