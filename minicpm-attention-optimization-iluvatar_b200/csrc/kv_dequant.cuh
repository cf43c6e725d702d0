// kv_dequant.cuh -- the pages a batch's block table references, from a
// quantised KV cache into a dense cache in the query dtype, for the tcgen05
// attention kernel.
//
// Attention over quantised caches is what the reference's service sends to
// vLLM's unified_attention (integration/vllm-plugin-FL-split-kv.patch:473-523
// sets up the per-token-head scale caches; vLLM 0.22
// vllm/v1/attention/ops/triton_unified_attention.py:39-55 and :469-511 give
// the arithmetic):
//   * fp8 per-tensor: an element is fp8(x) * scale, rounded to the query dtype
//     (_cast_kv_tile), with scale the first element of k_descale / v_descale;
//   * int8 / fp8 per-token-head: an element times the scale of its (block,
//     slot, head); vLLM folds that scale into S (keys) and P (values), here it
//     is applied to the element, rounded to the query dtype.
// Every element of a referenced page is converted, including the rows of the
// last page past the sequence end, which the attention kernel masks.  Page p
// of sequence b lands at dense page b * max_pages + p, and the dense block
// table gets that index; pages past a sequence's length get a table entry and
// no data.  A block id outside [0, num_blocks) gives a zero page.
//
// Bandwidth kernel: a persistent grid-stride loop over the dense pages; 8-byte
// loads and 16-byte stores when every cache row is 8-byte aligned, else 4-byte
// loads and 8-byte stores (the per-token-head rows carry their 4-byte scale
// inline, so they are only 4-byte aligned); four pieces per thread in flight
// before any is stored.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <type_traits>

#include "kv_cache_write.cuh"

namespace b200 {

constexpr int kDequantThreads = 256;

struct KvDequantArgs {
  const uint8_t* kc;
  const uint8_t* vc;
  int64_t kc_sb, kc_st, kc_sh, vc_sb, vc_st, vc_sh;  // byte strides of the 1-byte caches
  const float* k_scale;  // per-tensor
  const float* v_scale;
  const float* ksc;      // per-token-head, float strides
  const float* vsc;
  int64_t ks_sb, ks_st, ks_sh, vs_sb, vs_st, vs_sh;
  const void* block_table;
  int64_t bt_stride;
  int bt_cols, bt_i64;
  const void* seqused;
  int len_i64;
  void* out;       // [num_seqs * max_pages, 2, block_size, hkv, head_dim]
  int* out_table;  // [num_seqs, max_pages]
  int num_seqs, max_pages, block_size, hkv, head_dim, num_blocks;
};

template <int kElem>
__device__ __forceinline__ void decode4(uint32_t w, float (&f)[4]) {
  if (kElem == kElemI8) {
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = static_cast<float>(static_cast<int8_t>((w >> (8 * i)) & 0xff));
  } else {
    const __nv_fp8_interpretation_t fmt = kElem == kElemE4M3 ? __NV_E4M3 : __NV_E5M2;
    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xffff), fmt);
    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), fmt);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
}

template <typename T>
__device__ __forceinline__ uint2 encode4(const float (&f)[4]) {
  uint2 r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]), b = __floats2bfloat162_rn(f[2], f[3]);
    r.x = *reinterpret_cast<uint32_t*>(&a);
    r.y = *reinterpret_cast<uint32_t*>(&b);
  } else {
    __half2 a = __floats2half2_rn(f[0], f[1]), b = __floats2half2_rn(f[2], f[3]);
    r.x = *reinterpret_cast<uint32_t*>(&a);
    r.y = *reinterpret_cast<uint32_t*>(&b);
  }
  return r;
}

// A page: 2 (K, V) x block_size x hkv rows of head_dim elements, cut into
// pieces of kPiece elements (8 when every cache row is 8-byte aligned, else 4),
// consecutive threads on consecutive pieces, so a warp reads 128-256 and
// writes 256-512 contiguous bytes per instruction.  Persistent grid-stride loop over the dense pages; every thread loads
// its pieces of a page before converting and storing them.
template <typename T, int kElem, bool kPerTokenHead, int kPiece>
__global__ void __launch_bounds__(kDequantThreads) kv_dequant_kernel(const KvDequantArgs a) {
  constexpr int kPer = 4;  // pieces a thread keeps in flight per page
  const int pieces_per_row = a.head_dim / kPiece;
  const int per_cache = a.block_size * a.hkv * pieces_per_row;
  const int total_pages = a.num_seqs * a.max_pages;
  const float ks_tensor = kPerTokenHead ? 1.f : __ldg(a.k_scale);
  const float vs_tensor = kPerTokenHead ? 1.f : __ldg(a.v_scale);
  for (int dst_page = blockIdx.x; dst_page < total_pages; dst_page += gridDim.x) {
    const int b = dst_page / a.max_pages, p = dst_page - b * a.max_pages;
    if (threadIdx.x == 0) a.out_table[dst_page] = dst_page;
    const int L = static_cast<int>(kv_load_index(a.seqused, b, a.len_i64));
    if (p * a.block_size >= L || p >= a.bt_cols) continue;  // CTA-uniform
    const int64_t src = kv_load_index(a.block_table, static_cast<int64_t>(b) * a.bt_stride + p, a.bt_i64);
    const bool have = src >= 0 && src < a.num_blocks;
    T* out = static_cast<T*>(a.out) + static_cast<int64_t>(dst_page) * 2 * a.block_size * a.hkv * a.head_dim;
    for (int base = threadIdx.x; base < 2 * per_cache; base += kPer * kDequantThreads) {
      uint32_t w[kPer][kPiece / 4];
      float sc[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int i = base + k * kDequantThreads;
        sc[k] = 0.f;
#pragma unroll
        for (int e = 0; e < kPiece / 4; ++e) w[k][e] = 0u;
        if (i < 2 * per_cache && have) {
          const int kv = i >= per_cache;
          const int r = kv ? i - per_cache : i;
          const int piece = r % pieces_per_row, row = r / pieces_per_row;
          const int slot = row / a.hkv, head = row - slot * a.hkv;
          const uint8_t* src_row = (kv ? a.vc : a.kc) + src * (kv ? a.vc_sb : a.kc_sb) +
                                   slot * (kv ? a.vc_st : a.kc_st) + head * (kv ? a.vc_sh : a.kc_sh);
          if (kPiece == 8) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(src_row + 8 * piece));
            w[k][0] = v.x; w[k][1] = v.y;
          } else {
            w[k][0] = __ldg(reinterpret_cast<const uint32_t*>(src_row + 4 * piece));
          }
          if (kPerTokenHead) {
            sc[k] = kv ? __ldg(a.vsc + src * a.vs_sb + slot * a.vs_st + head * a.vs_sh)
                       : __ldg(a.ksc + src * a.ks_sb + slot * a.ks_st + head * a.ks_sh);
          } else {
            sc[k] = kv ? vs_tensor : ks_tensor;
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int i = base + k * kDequantThreads;
        if (i >= 2 * per_cache) break;
        const int kv = i >= per_cache;
        const int r = kv ? i - per_cache : i;
        const int piece = r % pieces_per_row, row = r / pieces_per_row;
        // dense page layout [2][block_size][hkv][head_dim]
        T* dst = out + (static_cast<int64_t>(kv) * a.block_size * a.hkv + row) * a.head_dim + kPiece * piece;
        uint2 enc[kPiece / 4];
#pragma unroll
        for (int e = 0; e < kPiece / 4; ++e) {
          float f[4];
          decode4<kElem>(w[k][e], f);
#pragma unroll
          for (int x = 0; x < 4; ++x) f[x] *= sc[k];
          enc[e] = encode4<T>(f);
        }
        if (kPiece == 8) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(enc[0].x, enc[0].y, enc[kPiece / 4 - 1].x, enc[kPiece / 4 - 1].y);
        } else {
          *reinterpret_cast<uint2*>(dst) = enc[0];
        }
      }
    }
  }
}

}  // namespace b200
