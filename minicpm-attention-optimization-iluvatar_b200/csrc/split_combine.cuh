// split_combine.cuh -- LSE-weighted combine of Split-KV partial outputs.
//
// Follows _split_kv_reduce (kernels/triton_split_kv_paged.py:197-228 of the
// reference project): m* = max_s m_s; w_s = exp(m_s - m*) * l_s when l_s > 0,
// else 0; out = sum_s w_s O_s / max(sum_s w_s, 1e-20).  A split with
// l_s == 0 contributes nothing (the reference multiplies it by 0; here it
// is selected out, so even a NaN there cannot reach the output).
//
// Bandwidth kernel: one (token, head) row per group of D/8 threads, each
// thread moving 8 elements of every split with 16-byte loads and stores.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100_ptx.cuh"

namespace b200 {

constexpr int kCombineThreads = 256;
constexpr int kMaxSplits = 16;

struct CombineArgs {
  const void* o;
  const float* m;
  const float* l;
  void* out;
  int64_t o_ss, o_st, o_sh;
  int64_t m_ss, m_st, m_sh;
  int64_t l_ss, l_st, l_sh;
  int64_t out_st, out_sh;
  int num_splits, total_q, num_heads;
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 w;
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 c = __floats2bfloat162_rn(v[4], v[5]), d = __floats2bfloat162_rn(v[6], v[7]);
  w.x = *reinterpret_cast<uint32_t*>(&a);
  w.y = *reinterpret_cast<uint32_t*>(&b);
  w.z = *reinterpret_cast<uint32_t*>(&c);
  w.w = *reinterpret_cast<uint32_t*>(&d);
  *reinterpret_cast<uint4*>(p) = w;
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
  uint4 w;
  __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
  __half2 c = __floats2half2_rn(v[4], v[5]), d = __floats2half2_rn(v[6], v[7]);
  w.x = *reinterpret_cast<uint32_t*>(&a);
  w.y = *reinterpret_cast<uint32_t*>(&b);
  w.z = *reinterpret_cast<uint32_t*>(&c);
  w.w = *reinterpret_cast<uint32_t*>(&d);
  *reinterpret_cast<uint4*>(p) = w;
}

// Raw 16-byte pieces of one row chunk of 8 elements (one piece for 16-bit
// types, two for fp32), loaded with the streaming hint: partials are read once.
template <typename T>
struct SplitChunk8 {
  static constexpr int kPieces = sizeof(T) == 4 ? 2 : 1;
  uint4 w[kPieces];
  __device__ __forceinline__ void load(const T* p) {
#pragma unroll
    for (int i = 0; i < kPieces; ++i) w[i] = __ldcs(reinterpret_cast<const uint4*>(p) + i);
  }
  __device__ __forceinline__ void to_float(float (&v)[8]) const;
};
template <>
__device__ __forceinline__ void SplitChunk8<float>::to_float(float (&v)[8]) const {
  v[0] = __uint_as_float(w[0].x); v[1] = __uint_as_float(w[0].y); v[2] = __uint_as_float(w[0].z); v[3] = __uint_as_float(w[0].w);
  v[4] = __uint_as_float(w[1].x); v[5] = __uint_as_float(w[1].y); v[6] = __uint_as_float(w[1].z); v[7] = __uint_as_float(w[1].w);
}
template <>
__device__ __forceinline__ void SplitChunk8<__nv_bfloat16>::to_float(float (&v)[8]) const {
  const uint32_t u[4] = {w[0].x, w[0].y, w[0].z, w[0].w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void SplitChunk8<__half>::to_float(float (&v)[8]) const {
  const uint32_t u[4] = {w[0].x, w[0].y, w[0].z, w[0].w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// One (token, head) row per D/8 threads, up to kS splits (kS = 4, 8 or 16,
// the smallest bound >= num_splits).  Every load of a row -- the partial
// O chunks of all splits and the m / l values -- is issued before any is
// used, so a row costs one memory round trip.  The m / l values of a row are
// loaded once per row group (thread j of the group holds splits j, j + D/8,
// ...), the group reduces the maximum and forms each split's weight, and the
// weights reach every thread of the group by shuffles.  A split with l = 0
// carries weight -1 and is left out by selection (its O, whatever it holds,
// never reaches the sum).  `o`, `m`, `l` point at split 0 of the row; every
// thread of the group calls this (the shuffles need all of them), and only
// threads with `valid` store.
template <typename TO, typename TOut, int D, int kS>
__device__ __forceinline__ void combine_row(const TO* o, int64_t o_ss, const float* m, int64_t m_ss, const float* l,
                                            int64_t l_ss, int num_splits, TOut* dst, bool valid) {
  constexpr int kThreadsPerRow = D / 8;
  constexpr int kPer = (kS + kThreadsPerRow - 1) / kThreadsPerRow;  // splits whose m / l one thread loads
  const int sub = threadIdx.x % kThreadsPerRow;
  const int d0 = sub * 8;
  SplitChunk8<TO> raw[kS];
#pragma unroll
  for (int s = 0; s < kS; ++s)
    if (s < num_splits) raw[s].load(o + s * o_ss + d0);
  float mk[kPer], lk[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int s = sub + k * kThreadsPerRow;
    mk[k] = -INFINITY;
    lk[k] = 0.f;
    if (s < num_splits) {
      mk[k] = __ldg(m + s * m_ss);
      lk[k] = __ldg(l + s * l_ss);
    }
  }
  float m_max = mk[0];
#pragma unroll
  for (int k = 1; k < kPer; ++k) m_max = fmaxf(m_max, mk[k]);
#pragma unroll
  for (int off = kThreadsPerRow / 2; off > 0; off >>= 1)
    m_max = fmaxf(m_max, __shfl_xor_sync(0xffffffffu, m_max, off, kThreadsPerRow));
  float wk[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) wk[k] = lk[k] > 0.f ? expf(mk[k] - m_max) * lk[k] : -1.f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float denom = 0.f;
#pragma unroll
  for (int s = 0; s < kS; ++s) {
    if (s < num_splits) {
      const float w = __shfl_sync(0xffffffffu, wk[s / kThreadsPerRow], s % kThreadsPerRow, kThreadsPerRow);
      if (w >= 0.f) {
        float v[8];
        raw[s].to_float(v);
        denom += w;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, v[i], acc[i]);
      }
    }
  }
  const float inv = 1.f / fmaxf(denom, 1e-20f);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] *= inv;
  if (valid) store8<TOut>(dst + d0, acc);
}

// The reduce of caller-supplied partials [S, T, H, D] (b200_split_combine).
template <typename TO, typename TOut, int D, int kS>
__global__ void __launch_bounds__(kCombineThreads) split_combine_kernel(const CombineArgs a) {
  constexpr int kThreadsPerRow = D / 8;
  constexpr int kRowsPerBlock = kCombineThreads / kThreadsPerRow;
  const int64_t nrows = static_cast<int64_t>(a.total_q) * a.num_heads;
  const int64_t row_raw = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + threadIdx.x / kThreadsPerRow;
  const bool valid = row_raw < nrows;  // threads past the end still take part in the shuffles
  const int64_t row = valid ? row_raw : nrows - 1;
  const int64_t t = row / a.num_heads;
  const int64_t h = row - t * a.num_heads;
  combine_row<TO, TOut, D, kS>(static_cast<const TO*>(a.o) + t * a.o_st + h * a.o_sh, a.o_ss,
                               a.m + t * a.m_st + h * a.m_sh, a.m_ss, a.l + t * a.l_st + h * a.l_sh, a.l_ss,
                               a.num_splits, static_cast<TOut*>(a.out) + t * a.out_st + h * a.out_sh, valid);
}

}  // namespace b200
