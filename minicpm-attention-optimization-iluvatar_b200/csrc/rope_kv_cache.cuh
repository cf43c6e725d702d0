// rope_kv_cache.cuh -- fused RoPE + paged KV-cache write.
//
// Semantics of _rope_and_cache_kernel (kernels/triton_rope_kv_cache.py:49-202
// of the reference project):
//   * cos_sin_cache[pos] = [cos(0..rd/2) | sin(0..rd/2)];
//   * NeoX pairs (d, d + rd/2), interleaved pairs (2i, 2i + 1);
//     first' = x1*cos - x2*sin, second' = x2*cos + x1*sin, in fp32, each
//     product rounded before the add (no fused multiply-add), then rounded
//     to the storage dtype (round to nearest even);
//   * dims >= rotary_dim pass through;
//   * Q is rotated in place for every token; rotated K and unchanged V go to
//     cache[slot / bs, slot % bs, h, :] unless slot < 0.
// Out-of-range indices, which the reference would read or write out of
// bounds, are skipped here and recorded in the device error word.
//
// The service variant (IluvatarAttentionImpl.do_rope_and_kv_cache_update,
// integration/vllm-plugin-FL-split-kv.patch:865-899, which passes
// k_out = key) additionally stores the rotated key of every token to key_out
// and may write fp8 caches: the value the cache receives is the one an
// unfused rotate-then-cache-update sequence would store, i.e. the rotated
// element rounded to the model dtype, divided by k_scale / v_scale (rounded
// to nearest) and converted to fp8 (RNE, saturating).
//
// Bandwidth kernel: one thread per 8-element unit (a NeoX unit is the chunk
// at d plus its partner chunk at d + rd/2), 16-byte loads and stores.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kv_cache_write.cuh"
#include "split_combine.cuh"

namespace b200 {

constexpr int kRopeThreads = 256;

struct RopeArgs {
  void* q;
  const void* k;
  const void* v;
  const void* pos;
  const void* cs;
  void* kc;
  void* vc;
  const void* slot;
  int64_t q_st, q_sh, q_sd;
  int64_t k_st, k_sh, k_sd;
  int64_t v_st, v_sh, v_sd;
  int64_t cs_st;
  int64_t c_sb, c_st, c_sh, c_sd;
  int64_t num_slots;
  int num_tokens, hq, hkv, head_dim, rd, block_size, max_position;
  int pos_i64, slot_i64;
  // Service variant only.
  void* ko;
  int64_t ko_st, ko_sh;
  int cache_elem;  // KvCacheElem: kElemSame, kElemE4M3 or kElemE5M2
  const float* k_scale;
  const float* v_scale;
};

__device__ __forceinline__ int64_t load_i(const void* p, int64_t i, int is_i64) {
  return is_i64 ? static_cast<const int64_t*>(p)[i] : static_cast<int64_t>(static_cast<const int*>(p)[i]);
}

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 a = *reinterpret_cast<const uint2*>(p);
  const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
  const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
  v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
}
template <>
__device__ __forceinline__ void load4<__half>(const __half* p, float (&v)[4]) {
  const uint2 a = *reinterpret_cast<const uint2*>(p);
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&a.x));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&a.y));
  v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// first' = a*c - b*s ; second' = b*c + a*s, products rounded separately.
__device__ __forceinline__ void rotate_pair(float a, float b, float c, float s, float& ra, float& rb) {
  ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  rb = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

// Vector path: d contiguous and 16-byte aligned rows; rd % 16 == 0 (NeoX) or rd % 8 == 0.
template <typename T, typename CS, bool NEOX>
__global__ void __launch_bounds__(kRopeThreads) rope_kv_vec_kernel(const RopeArgs a) {
  const int half = a.rd / 2;
  const int n_rot = NEOX ? half / 8 : a.rd / 8;  // rotation units per head
  const int n_pass = (a.head_dim - a.rd) / 8;     // K pass-through chunks per head
  const int n_v = a.head_dim / 8;                 // V chunks per head
  const int q_items = a.hq * n_rot;
  const int k_items = a.hkv * (n_rot + n_pass);
  const int per_token = q_items + k_items + a.hkv * n_v;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t token = gid / per_token;
  if (token >= a.num_tokens) return;
  int item = static_cast<int>(gid - token * per_token);

  const int64_t pos = load_i(a.pos, token, a.pos_i64);
  if (pos < 0 || pos >= a.max_position) {
    if (item == 0) record_device_error(B200_DEVERR_POS_RANGE);
    return;
  }
  const CS* cs_row = static_cast<const CS*>(a.cs) + pos * a.cs_st;

  if (item < q_items) {
    const int h = item / n_rot, u = item - h * n_rot;
    T* qrow = static_cast<T*>(a.q) + token * a.q_st + h * a.q_sh;
    if (NEOX) {
      float x1[8], x2[8], c[8], s[8];
      load8<T>(qrow + 8 * u, x1);
      load8<T>(qrow + half + 8 * u, x2);
      load8<CS>(cs_row + 8 * u, c);
      load8<CS>(cs_row + half + 8 * u, s);
      float y1[8], y2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) rotate_pair(x1[i], x2[i], c[i], s[i], y1[i], y2[i]);
      store8<T>(qrow + 8 * u, y1);
      store8<T>(qrow + half + 8 * u, y2);
    } else {
      float x[8], c[4], s[4], y[8];
      load8<T>(qrow + 8 * u, x);
      load4<CS>(cs_row + 4 * u, c);
      load4<CS>(cs_row + half + 4 * u, s);
#pragma unroll
      for (int i = 0; i < 4; ++i) rotate_pair(x[2 * i], x[2 * i + 1], c[i], s[i], y[2 * i], y[2 * i + 1]);
      store8<T>(qrow + 8 * u, y);
    }
    return;
  }
  item -= q_items;

  const int64_t slot = load_i(a.slot, token, a.slot_i64);
  if (slot < 0) return;
  if (slot >= a.num_slots) {
    if (item == 0) record_device_error(B200_DEVERR_SLOT_RANGE);
    return;
  }
  const int64_t blk = slot / a.block_size, off = slot - blk * a.block_size;

  if (item < k_items) {
    const int per_head = n_rot + n_pass;
    const int h = item / per_head, u = item - h * per_head;
    const T* krow = static_cast<const T*>(a.k) + token * a.k_st + h * a.k_sh;
    T* crow = static_cast<T*>(a.kc) + blk * a.c_sb + off * a.c_st + h * a.c_sh;
    if (u >= n_rot) {  // pass-through chunk
      const int d = a.rd + 8 * (u - n_rot);
      *reinterpret_cast<uint4*>(crow + d) = *reinterpret_cast<const uint4*>(krow + d);
      return;
    }
    if (NEOX) {
      float x1[8], x2[8], c[8], s[8], y1[8], y2[8];
      load8<T>(krow + 8 * u, x1);
      load8<T>(krow + half + 8 * u, x2);
      load8<CS>(cs_row + 8 * u, c);
      load8<CS>(cs_row + half + 8 * u, s);
#pragma unroll
      for (int i = 0; i < 8; ++i) rotate_pair(x1[i], x2[i], c[i], s[i], y1[i], y2[i]);
      store8<T>(crow + 8 * u, y1);
      store8<T>(crow + half + 8 * u, y2);
    } else {
      float x[8], c[4], s[4], y[8];
      load8<T>(krow + 8 * u, x);
      load4<CS>(cs_row + 4 * u, c);
      load4<CS>(cs_row + half + 4 * u, s);
#pragma unroll
      for (int i = 0; i < 4; ++i) rotate_pair(x[2 * i], x[2 * i + 1], c[i], s[i], y[2 * i], y[2 * i + 1]);
      store8<T>(crow + 8 * u, y);
    }
    return;
  }
  item -= k_items;
  const int h = item / n_v, u = item - h * n_v;
  const T* vrow = static_cast<const T*>(a.v) + token * a.v_st + h * a.v_sh;
  T* crow = static_cast<T*>(a.vc) + blk * a.c_sb + off * a.c_st + h * a.c_sh;
  *reinterpret_cast<uint4*>(crow + 8 * u) = *reinterpret_cast<const uint4*>(vrow + 8 * u);
}

// Element path for any strides: one thread per rotation pair or copied element.
template <typename T, typename CS>
__global__ void __launch_bounds__(kRopeThreads) rope_kv_scalar_kernel(const RopeArgs a, const int neox) {
  const int half = a.rd / 2;
  const int q_items = a.hq * half;
  const int k_items = a.hkv * (half + (a.head_dim - a.rd));
  const int per_token = q_items + k_items + a.hkv * a.head_dim;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t token = gid / per_token;
  if (token >= a.num_tokens) return;
  int item = static_cast<int>(gid - token * per_token);
  const int64_t pos = load_i(a.pos, token, a.pos_i64);
  if (pos < 0 || pos >= a.max_position) {
    if (item == 0) record_device_error(B200_DEVERR_POS_RANGE);
    return;
  }
  const CS* cs_row = static_cast<const CS*>(a.cs) + pos * a.cs_st;
  auto pair_dims = [&](int i, int& d1, int& d2) {
    if (neox) { d1 = i; d2 = i + half; } else { d1 = 2 * i; d2 = 2 * i + 1; }
  };
  if (item < q_items) {
    const int h = item / half, i = item - h * half;
    int d1, d2;
    pair_dims(i, d1, d2);
    T* qrow = static_cast<T*>(a.q) + token * a.q_st + h * a.q_sh;
    float y1, y2;
    rotate_pair(to_f32(qrow[d1 * a.q_sd]), to_f32(qrow[d2 * a.q_sd]), to_f32(cs_row[i]), to_f32(cs_row[half + i]), y1, y2);
    qrow[d1 * a.q_sd] = from_f32<T>(y1);
    qrow[d2 * a.q_sd] = from_f32<T>(y2);
    return;
  }
  item -= q_items;
  const int64_t slot = load_i(a.slot, token, a.slot_i64);
  if (slot < 0) return;
  if (slot >= a.num_slots) {
    if (item == 0) record_device_error(B200_DEVERR_SLOT_RANGE);
    return;
  }
  const int64_t blk = slot / a.block_size, off = slot - blk * a.block_size;
  if (item < k_items) {
    const int per_head = half + (a.head_dim - a.rd);
    const int h = item / per_head, u = item - h * per_head;
    const T* krow = static_cast<const T*>(a.k) + token * a.k_st + h * a.k_sh;
    T* crow = static_cast<T*>(a.kc) + blk * a.c_sb + off * a.c_st + h * a.c_sh;
    if (u >= half) {
      const int d = a.rd + (u - half);
      crow[d * a.c_sd] = krow[d * a.k_sd];
      return;
    }
    int d1, d2;
    pair_dims(u, d1, d2);
    float y1, y2;
    rotate_pair(to_f32(krow[d1 * a.k_sd]), to_f32(krow[d2 * a.k_sd]), to_f32(cs_row[u]), to_f32(cs_row[half + u]), y1, y2);
    crow[d1 * a.c_sd] = from_f32<T>(y1);
    crow[d2 * a.c_sd] = from_f32<T>(y2);
    return;
  }
  item -= k_items;
  const int h = item / a.head_dim, d = item - h * a.head_dim;
  const T* vrow = static_cast<const T*>(a.v) + token * a.v_st + h * a.v_sh;
  T* crow = static_cast<T*>(a.vc) + blk * a.c_sb + off * a.c_st + h * a.c_sh;
  crow[d * a.c_sd] = vrow[d * a.v_sd];
}

// Warp-per-token path for the common shapes: lane l owns rotation unit
// c = l % NC of every head (NC units per head, 32 % NC == 0), so it loads its
// cos/sin chunk once per token and reuses it for all query and key heads.
// The loads that do not depend on the position (a batch of query heads, the
// key and value rows) are issued before the cos/sin row, and the next
// token's position and slot are fetched a token ahead.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  load8<T>(reinterpret_cast<const T*>(&u), v);
}

// Eight rotated values (fp32) to a cache row: the model dtype, or fp8 of the
// value rounded to the model dtype and divided by the cache's scale.
template <typename T>
__device__ __forceinline__ void cache_store8(void* base, int64_t off, const float (&y)[8], int elem,
                                             const FixedDivisor& scale) {
  if (elem == kElemSame) {
    store8<T>(static_cast<T*>(base) + off, y);
    return;
  }
  float r[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) r[i] = to_f32<T>(from_f32<T>(y[i]));
  uint8_t* p = static_cast<uint8_t*>(base) + off;
  if (elem == kElemE4M3) store_fp8_scaled<kElemE4M3>(p, r, scale);
  else store_fp8_scaled<kElemE5M2>(p, r, scale);
}

// Eight unrotated elements (raw) to a cache row.
template <typename T>
__device__ __forceinline__ void cache_copy8(void* base, int64_t off, const uint4& x, int elem,
                                            const FixedDivisor& scale) {
  if (elem == kElemSame) {
    *reinterpret_cast<uint4*>(static_cast<T*>(base) + off) = x;
    return;
  }
  float v[8];
  load8<T>(reinterpret_cast<const T*>(&x), v);
  uint8_t* p = static_cast<uint8_t*>(base) + off;
  if (elem == kElemE4M3) store_fp8_scaled<kElemE4M3>(p, v, scale);
  else store_fp8_scaled<kElemE5M2>(p, v, scale);
}

// SVC = the service variant (key_out and / or an fp8 cache); SVC = false is
// the reference operator's path.
template <typename T, typename CS, bool NEOX, int NC, bool SVC>
__global__ void __launch_bounds__(kRopeThreads, 2) rope_kv_warp_kernel(const RopeArgs a) {
  constexpr int kHeadStep = 32 / NC;
  // Query heads per lane whose loads are in flight together: eight 16-byte
  // loads per lane either way (NeoX units span two chunks).
  constexpr int kQBatch = NEOX ? 4 : 8;
  const int lane = threadIdx.x & 31;
  const int c = lane % NC, hg = lane / NC;
  const int half = a.rd / 2;
  const int n_pass = (a.head_dim - a.rd) / 8;
  const int n_v = a.head_dim / 8;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  int64_t token = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  // The next token's position and slot are fetched one iteration ahead.
  int64_t pos_n = 0, slot_n = -1;
  if (token < a.num_tokens) {
    pos_n = load_i(a.pos, token, a.pos_i64);
    slot_n = load_i(a.slot, token, a.slot_i64);
  }
  for (; token < a.num_tokens; token += nwarps) {
    const int64_t pos = pos_n, slot = slot_n;
    if (token + nwarps < a.num_tokens) {
      pos_n = load_i(a.pos, token + nwarps, a.pos_i64);
      slot_n = load_i(a.slot, token + nwarps, a.slot_i64);
    }
    T* qtok = static_cast<T*>(a.q) + token * a.q_st;
    const T* ktok = static_cast<const T*>(a.k) + token * a.k_st;
    const T* vtok = static_cast<const T*>(a.v) + token * a.v_st;
    // Issue this token's loads that do not depend on the position first.
    uint4 q1[kQBatch], q2[kQBatch], k1, k2, vv;
#pragma unroll
    for (int k = 0; k < kQBatch; ++k) {
      const int h = hg + k * kHeadStep;
      if (h < a.hq) {
        q1[k] = *reinterpret_cast<const uint4*>(qtok + h * a.q_sh + 8 * c);
        if (NEOX) q2[k] = *reinterpret_cast<const uint4*>(qtok + h * a.q_sh + half + 8 * c);
      }
    }
    const bool k_lane = hg < a.hkv;
    if (k_lane) {
      k1 = *reinterpret_cast<const uint4*>(ktok + hg * a.k_sh + 8 * c);
      if (NEOX) k2 = *reinterpret_cast<const uint4*>(ktok + hg * a.k_sh + half + 8 * c);
    }
    const bool v_lane = lane < a.hkv * n_v;
    if (v_lane) vv = *reinterpret_cast<const uint4*>(vtok + (lane / n_v) * a.v_sh + 8 * (lane % n_v));

    if (pos < 0 || pos >= a.max_position) {
      if (lane == 0) record_device_error(B200_DEVERR_POS_RANGE);
      continue;
    }
    const CS* cs_row = static_cast<const CS*>(a.cs) + pos * a.cs_st;
    float cv[8], sv[8];
    if (NEOX) {
      load8<CS>(cs_row + 8 * c, cv);
      load8<CS>(cs_row + half + 8 * c, sv);
    } else {
      float c4[4], s4[4];
      load4<CS>(cs_row + 4 * c, c4);
      load4<CS>(cs_row + half + 4 * c, s4);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        cv[i] = c4[i];
        sv[i] = s4[i];
      }
    }
    auto rotate_store = [&](const uint4& x1, const uint4& x2, T* row) {
      float v1[8], y1[8];
      unpack8<T>(x1, v1);
      if (NEOX) {
        float v2[8], y2[8];
        unpack8<T>(x2, v2);
#pragma unroll
        for (int i = 0; i < 8; ++i) rotate_pair(v1[i], v2[i], cv[i], sv[i], y1[i], y2[i]);
        store8<T>(row + 8 * c, y1);
        store8<T>(row + half + 8 * c, y2);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) rotate_pair(v1[2 * i], v1[2 * i + 1], cv[i], sv[i], y1[2 * i], y1[2 * i + 1]);
        store8<T>(row + 8 * c, y1);
      }
    };
#pragma unroll
    for (int k = 0; k < kQBatch; ++k) {
      const int h = hg + k * kHeadStep;
      if (h < a.hq) rotate_store(q1[k], q2[k], qtok + h * a.q_sh);
    }
    // Query heads beyond the first batch, a batch of loads at a time.
    for (int h0 = hg + kQBatch * kHeadStep; h0 < a.hq; h0 += kQBatch * kHeadStep) {
#pragma unroll
      for (int k = 0; k < kQBatch; ++k) {
        const int h = h0 + k * kHeadStep;
        if (h < a.hq) {
          q1[k] = *reinterpret_cast<const uint4*>(qtok + h * a.q_sh + 8 * c);
          if (NEOX) q2[k] = *reinterpret_cast<const uint4*>(qtok + h * a.q_sh + half + 8 * c);
        }
      }
#pragma unroll
      for (int k = 0; k < kQBatch; ++k) {
        const int h = h0 + k * kHeadStep;
        if (h < a.hq) rotate_store(q1[k], q2[k], qtok + h * a.q_sh);
      }
    }
    if (SVC) {
      // Rotated key to key_out for every token; caches only for valid slots.
      const bool in_range = slot >= 0 && slot < a.num_slots;
      if (slot >= a.num_slots && lane == 0) record_device_error(B200_DEVERR_SLOT_RANGE);
      int64_t ctok = 0;
      if (in_range) {
        const int64_t blk = slot / a.block_size;
        ctok = blk * a.c_sb + (slot - blk * a.block_size) * a.c_st;
      }
      FixedDivisor ks{}, vs{};
      if (a.cache_elem != kElemSame) {
        ks = make_divisor(*a.k_scale);
        vs = make_divisor(*a.v_scale);
      }
      T* kotok = a.ko ? static_cast<T*>(a.ko) + token * a.ko_st : nullptr;
      auto rotate_key = [&](const uint4& x1, const uint4& x2, int h) {
        float v1[8], y1[8], y2[8];
        unpack8<T>(x1, v1);
        if (NEOX) {
          float v2[8];
          unpack8<T>(x2, v2);
#pragma unroll
          for (int i = 0; i < 8; ++i) rotate_pair(v1[i], v2[i], cv[i], sv[i], y1[i], y2[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) rotate_pair(v1[2 * i], v1[2 * i + 1], cv[i], sv[i], y1[2 * i], y1[2 * i + 1]);
        }
        if (kotok) {
          store8<T>(kotok + h * a.ko_sh + 8 * c, y1);
          if (NEOX) store8<T>(kotok + h * a.ko_sh + half + 8 * c, y2);
        }
        if (in_range) {
          cache_store8<T>(a.kc, ctok + h * a.c_sh + 8 * c, y1, a.cache_elem, ks);
          if (NEOX) cache_store8<T>(a.kc, ctok + h * a.c_sh + half + 8 * c, y2, a.cache_elem, ks);
        }
      };
      if (k_lane) rotate_key(k1, k2, hg);
      for (int h = hg + kHeadStep; h < a.hkv; h += kHeadStep) {
        const uint4 x1 = *reinterpret_cast<const uint4*>(ktok + h * a.k_sh + 8 * c);
        const uint4 x2 = NEOX ? *reinterpret_cast<const uint4*>(ktok + h * a.k_sh + half + 8 * c) : x1;
        rotate_key(x1, x2, h);
      }
      const bool ko_copy = kotok && a.ko != a.k;  // pass-through dims of an in-place key_out stay as they are
      for (int i = lane; i < a.hkv * n_pass; i += 32) {
        const int h = i / n_pass, d = a.rd + 8 * (i - h * n_pass);
        const uint4 x = *reinterpret_cast<const uint4*>(ktok + h * a.k_sh + d);
        if (ko_copy) *reinterpret_cast<uint4*>(kotok + h * a.ko_sh + d) = x;
        if (in_range) cache_copy8<T>(a.kc, ctok + h * a.c_sh + d, x, a.cache_elem, ks);
      }
      if (in_range) {
        if (v_lane) cache_copy8<T>(a.vc, ctok + (lane / n_v) * a.c_sh + 8 * (lane % n_v), vv, a.cache_elem, vs);
        for (int i = lane + 32; i < a.hkv * n_v; i += 32) {
          const int h = i / n_v, d = 8 * (i - h * n_v);
          cache_copy8<T>(a.vc, ctok + h * a.c_sh + d, *reinterpret_cast<const uint4*>(vtok + h * a.v_sh + d),
                         a.cache_elem, vs);
        }
      }
      continue;
    }
    if (slot < 0) continue;
    if (slot >= a.num_slots) {
      if (lane == 0) record_device_error(B200_DEVERR_SLOT_RANGE);
      continue;
    }
    const int64_t blk = slot / a.block_size, off = slot - blk * a.block_size;
    T* kc_tok = static_cast<T*>(a.kc) + blk * a.c_sb + off * a.c_st;
    T* vc_tok = static_cast<T*>(a.vc) + blk * a.c_sb + off * a.c_st;
    if (k_lane) rotate_store(k1, k2, kc_tok + hg * a.c_sh);
    for (int h = hg + kHeadStep; h < a.hkv; h += kHeadStep) {
      const uint4 x1 = *reinterpret_cast<const uint4*>(ktok + h * a.k_sh + 8 * c);
      const uint4 x2 = NEOX ? *reinterpret_cast<const uint4*>(ktok + h * a.k_sh + half + 8 * c) : x1;
      rotate_store(x1, x2, kc_tok + h * a.c_sh);
    }
    for (int i = lane; i < a.hkv * n_pass; i += 32) {
      const int h = i / n_pass, d = a.rd + 8 * (i - h * n_pass);
      *reinterpret_cast<uint4*>(kc_tok + h * a.c_sh + d) = *reinterpret_cast<const uint4*>(ktok + h * a.k_sh + d);
    }
    if (v_lane) *reinterpret_cast<uint4*>(vc_tok + (lane / n_v) * a.c_sh + 8 * (lane % n_v)) = vv;
    for (int i = lane + 32; i < a.hkv * n_v; i += 32) {
      const int h = i / n_v, d = 8 * (i - h * n_v);
      *reinterpret_cast<uint4*>(vc_tok + h * a.c_sh + d) = *reinterpret_cast<const uint4*>(vtok + h * a.v_sh + d);
    }
  }
}

}  // namespace b200
