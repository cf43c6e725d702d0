/*
 * minicpm_b200.h -- C ABI of the sm_100a paged prefill attention and the
 * fused RoPE + paged KV-cache write.
 *
 * Plain C: device pointers, element strides and sizes; no framework types.
 * Every entry point returns a status code (B200_OK on success) and never
 * throws; b200_last_error() gives the message of the last failure on the
 * calling thread.  All work is enqueued on the given CUDA stream
 * (a cudaStream_t passed as void*; NULL is the legacy default stream) and
 * no entry point synchronises the host, allocates device memory or
 * launches anything on another stream.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   b200_paged_attn_fwd    -> the two launches of paged_split_kv_attention,
 *                             kernels/triton_split_kv_paged.py:283-360
 *                             (_split_kv_forward :18-155, _split_kv_reduce
 *                             :158-228), including the q-block compaction
 *                             (:283-293) that the reference does on the host.
 *   b200_split_combine     -> the _split_kv_reduce launch on its own,
 *                             kernels/triton_split_kv_paged.py:342-360.
 *   b200_rope_kv_write     -> the _rope_and_cache_kernel launch of
 *                             fused_rope_and_cache,
 *                             kernels/triton_rope_kv_cache.py:261-286.
 *   b200_choose_num_splits -> the fixed split count of
 *                             kernels/attention.py:166 and
 *                             kernels/triton_unified_attention_optimized.py:216-218
 *                             (the reference has no automatic choice).
 *   b200_attn_workspace_bytes -> the per-call scratch allocation of
 *                             kernels/triton_split_kv_paged.py:295-306.
 *   b200_kv_cache_write    -> the service's plain KV-cache update,
 *                             IluvatarAttentionImpl.do_kv_cache_update
 *                             (integration/vllm-plugin-FL-split-kv.patch:815-858),
 *                             i.e. vLLM's triton_reshape_and_cache_flash and
 *                             triton_reshape_and_cache_flash_per_token_head_quant.
 *   b200_rope_kv_write with key_out / an fp8 cache
 *                          -> the service RoPE ABI,
 *                             IluvatarAttentionImpl.do_rope_and_kv_cache_update
 *                             (integration/vllm-plugin-FL-split-kv.patch:865-899).
 */
#ifndef MINICPM_B200_H_
#define MINICPM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_ABI_VERSION 2

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

/* Status codes. */
#define B200_OK 0
#define B200_ERR_INVALID 1     /* bad shape, stride, dtype or argument value  */
#define B200_ERR_UNSUPPORTED 2 /* valid for the reference, not for this build */
#define B200_ERR_CUDA 3        /* a CUDA runtime / driver call failed          */
#define B200_ERR_WORKSPACE 4   /* workspace missing or too small               */

/* Element types. */
#define B200_DTYPE_F16 0
#define B200_DTYPE_BF16 1
#define B200_DTYPE_F32 2
#define B200_DTYPE_I32 3
#define B200_DTYPE_I64 4
#define B200_DTYPE_FP8_E4M3 5 /* cache element types of the quantised KV-cache writes */
#define B200_DTYPE_FP8_E5M2 6
#define B200_DTYPE_I8 7

/* KV-cache quantisation modes (same numbering as vLLM's KVQuantMode). */
#define B200_KVQ_NONE 0               /* cache dtype == key dtype: bit copy                */
#define B200_KVQ_FP8_PER_TENSOR 1     /* fp8(x / scale), one device float per cache        */
#define B200_KVQ_INT8_PER_TOKEN_HEAD 2 /* int8 with a dynamic scale per (token, head)      */
#define B200_KVQ_FP8_PER_TOKEN_HEAD 3  /* fp8 e4m3 with a dynamic scale per (token, head)  */

/* Device-side error codes (b200_device_error). */
#define B200_DEVERR_NONE 0u
#define B200_DEVERR_WAIT_TIMEOUT 1u /* an in-kernel wait ran past its limit     */
#define B200_DEVERR_SLOT_RANGE 2u   /* slot_mapping entry >= num_blocks*bs      */
#define B200_DEVERR_POS_RANGE 3u    /* position outside the cos/sin table        */
#define B200_DEVERR_DECODE_QLEN 4u  /* max_seqlen_q = 1 but a sequence has more query tokens */

/*
 * Paged causal varlen attention (prefill / chunked prefill), GQA, Split-KV.
 *
 * q          [total_q, num_q_heads, head_dim], element strides q_stride_t/h, d contiguous
 * k, v       paged caches [num_blocks, block_size, num_kv_heads, head_dim], strides
 *            *_stride_block/_tok/_head, d contiguous (the cache[:, 0] / cache[:, 1]
 *            views of a [num_blocks, 2, block_size, KH, D] cache are accepted)
 * out        [total_q, num_q_heads, head_dim], written in place
 * block_table [num_seqs, block_table_cols], int32 or int64, row stride in elements
 * cu_seqlens_q [num_seqs + 1], seqused_k [num_seqs]: int32 or int64
 * num_splits  0 = choose automatically, else 1..16.  A decode batch (max_seqlen_q == 1)
 *             runs the decode kernel, which splits the keys of each sequence into
 *             chunks of its own choosing; num_splits does not change the result.
 * workspace   device buffer of at least b200_attn_workspace_bytes(...) bytes,
 *             owned by the caller; must not be shared by calls that overlap.
 * All pointers: 16-byte aligned; all strides except d: multiples of 8 elements.
 */
typedef struct B200AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  const void* block_table;
  const void* cu_seqlens_q;
  const void* seqused_k;
  int64_t q_stride_t, q_stride_h;
  int64_t k_stride_block, k_stride_tok, k_stride_head;
  int64_t v_stride_block, v_stride_tok, v_stride_head;
  int64_t out_stride_t, out_stride_h;
  int64_t block_table_stride;
  int32_t block_table_cols;
  int32_t block_table_dtype; /* B200_DTYPE_I32 / I64 */
  int32_t seqlen_dtype;      /* dtype of cu_seqlens_q and seqused_k: I32 / I64 */
  int32_t dtype;             /* q / k / v / out element type: F16 / BF16 */
  int32_t num_seqs;
  int32_t total_q;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t block_size;
  int32_t num_blocks;
  int32_t max_seqlen_q;
  int32_t max_seqlen_k;
  int32_t num_splits;
  float softmax_scale;
  void* workspace;
  size_t workspace_bytes;
} B200AttnParams;

/* Workspace bytes b200_paged_attn_fwd needs for these sizes (num_splits 0 = auto). */
B200_API size_t b200_attn_workspace_bytes(int32_t total_q, int32_t num_seqs, int32_t num_q_heads,
                                 int32_t num_kv_heads, int32_t head_dim, int32_t num_splits,
                                 int32_t max_seqlen_k, int32_t dtype);

/* The split count b200_paged_attn_fwd uses for num_splits = 0. */
B200_API int32_t b200_choose_num_splits(int32_t total_q, int32_t num_seqs, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t max_seqlen_k);

B200_API int b200_paged_attn_fwd(const B200AttnParams* params, void* stream);

/*
 * 1 if b200_paged_attn_fwd runs this head shape and element type, else 0:
 * q/k/v/out F16 or BF16, head_dim 64, 128 or 256, num_q_heads a multiple of
 * num_kv_heads with at most 128 query heads per KV head.  The dispatcher and
 * the service route other shapes to their baseline kernel before calling in,
 * as they route the unsupported features of kernels/attention.py:99-110 and
 * integration/vllm-plugin-FL-split-kv.patch:88-141 (the reference's Triton
 * kernel takes head_dim 64/128/256 and any ratio,
 * kernels/triton_split_kv_paged.py:270-279).
 */
B200_API int32_t b200_attn_shape_supported(int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                           int32_t dtype);

/*
 * b200_paged_attn_fwd without a caller-supplied workspace: no counterpart in
 * the reference.  For callers that cannot allocate device memory at call time
 * (an engine that reserved HBM for its KV cache up front, a foreign-language
 * host without a device allocator, a path where cudaMalloc's implicit device
 * synchronisation is not acceptable).  params->workspace and
 * params->workspace_bytes are ignored; the scratch is one file-scope device
 * array of B200_STATIC_SCRATCH_BYTES, held by every GPU that loads this
 * library until the process exits.  Calls whose scratch need
 * (b200_attn_workspace_bytes) exceeds it fail with B200_ERR_INVALID.  The
 * first call on a device looks up the array's device address (make it before
 * any stream capture) and keeps it for the life of the process: after a
 * cudaDeviceReset (or anything else that destroys the device's primary
 * context) that address is stale, so do not use this entry point across a
 * device reset.  All calls on a device share the array: calls that
 * overlap on the GPU (other streams, other threads) race and must not be
 * issued.  No scratch byte needs to start at zero; every byte a call reads
 * it wrote first.  Allocates nothing.
 */
#define B200_STATIC_SCRATCH_BYTES (32u << 20)
B200_API int b200_paged_attn_fwd_noalloc(const B200AttnParams* params, void* stream);

/*
 * Cross-split combine: out[t,h,:] = sum_s w_s O_s[t,h,:] / max(sum_s w_s, 1e-20),
 * w_s = exp(m_s - max_s m_s) * l_s for l_s > 0, else 0.
 * o_splits [num_splits, total_q, num_heads, head_dim] (F16 / BF16 / F32), m, l
 * [num_splits, total_q, num_heads] F32, out [total_q, num_heads, head_dim]
 * (F16 / BF16 / F32); d contiguous everywhere.
 */
typedef struct B200CombineParams {
  const void* o_splits;
  const float* m_splits;
  const float* l_splits;
  void* out;
  int64_t o_stride_s, o_stride_t, o_stride_h;
  int64_t m_stride_s, m_stride_t, m_stride_h;
  int64_t l_stride_s, l_stride_t, l_stride_h;
  int64_t out_stride_t, out_stride_h;
  int32_t o_dtype;
  int32_t out_dtype;
  int32_t num_splits;
  int32_t total_q;
  int32_t num_heads;
  int32_t head_dim;
} B200CombineParams;

B200_API int b200_split_combine(const B200CombineParams* params, void* stream);

/*
 * Fused RoPE + paged KV-cache write.  query [T, Hq, D] rotated in place;
 * rotate(key) -> key_cache[slot / bs, slot % bs, h, :]; value -> value_cache[...];
 * tokens with slot < 0 skip both cache writes.  cos_sin_cache [max_position,
 * rotary_dim] = [cos(0..rd/2) | sin(0..rd/2)].  Caches [num_blocks, bs, Hkv, D].
 */
typedef struct B200RopeParams {
  void* query;
  const void* key;
  const void* value;
  const void* positions;
  const void* cos_sin_cache;
  void* key_cache;
  void* value_cache;
  const void* slot_mapping;
  int64_t q_stride_t, q_stride_h, q_stride_d;
  int64_t k_stride_t, k_stride_h, k_stride_d;
  int64_t v_stride_t, v_stride_h, v_stride_d;
  int64_t cos_sin_stride_t;
  int64_t cache_stride_block, cache_stride_tok, cache_stride_head, cache_stride_d;
  int32_t num_tokens;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t rotary_dim;
  int32_t block_size;
  int32_t num_blocks;
  int32_t max_position;
  int32_t is_neox;
  int32_t dtype;          /* query / key / value / caches: F16 / BF16 */
  int32_t cos_sin_dtype;  /* F16 / BF16 / F32 */
  int32_t position_dtype; /* I32 / I64 */
  int32_t slot_dtype;     /* I32 / I64 */
  /* Service ABI (vLLM's rope-and-cache call with k_out = key):            */
  void* key_out;          /* NULL: key untouched; else rotated key [T, Hkv, D] stored here
                             for every token (may alias key)                             */
  int64_t ko_stride_t, ko_stride_h;
  int32_t cache_dtype;    /* == dtype, or FP8_E4M3 / FP8_E5M2: caches hold
                             fp8(round_to_dtype(x) / scale), RNE, saturating             */
  const float* k_scale;   /* fp8 caches: one device float each                           */
  const float* v_scale;
} B200RopeParams;

B200_API int b200_rope_kv_write(const B200RopeParams* params, void* stream);

/*
 * Paged KV-cache write (vLLM "flash" layout): for every token t with
 * slot_mapping[t] >= 0, key[t, h, :] -> key_cache[slot / bs, slot % bs, h, :]
 * and value[t, h, :] -> value_cache[...], as
 *   B200_KVQ_NONE                bit copy (cache_dtype == dtype);
 *   B200_KVQ_FP8_PER_TENSOR      fp8(x / *k_scale) (resp. *v_scale), x / s rounded to
 *                                nearest, fp8 round-to-nearest-even, saturating to the
 *                                largest finite value;
 *   B200_KVQ_*_PER_TOKEN_HEAD    s = max(max_d |x| / QMAX, 1e-6) per (token, head),
 *                                q = clamp(x * (1 / s), QMIN, QMAX) -> int8 by truncation
 *                                toward zero (QMAX 127, QMIN -128) or fp8 e4m3 RNE (±448);
 *                                s stored to k_scale_cache / v_scale_cache
 *                                [num_blocks, block_size, num_kv_heads] (float strides).
 * key, value [num_tokens, num_kv_heads, head_dim] (F16 / BF16 / F32), d contiguous;
 * caches [num_blocks, block_size, num_kv_heads, >= head_dim], d contiguous (the
 * per-token-head caches may carry the scale inline after head_dim).  Slots
 * >= num_blocks * block_size are skipped and recorded (B200_DEVERR_SLOT_RANGE).
 * Alignment: key / value rows 16 bytes; cache rows 16 bytes (NONE), 4 bytes (1-byte types).
 */
typedef struct B200KvWriteParams {
  const void* key;
  const void* value;
  void* key_cache;
  void* value_cache;
  const void* slot_mapping;
  const float* k_scale;  /* FP8_PER_TENSOR */
  const float* v_scale;
  float* k_scale_cache;  /* *_PER_TOKEN_HEAD */
  float* v_scale_cache;
  int64_t k_stride_t, k_stride_h;
  int64_t v_stride_t, v_stride_h;
  int64_t kc_stride_block, kc_stride_tok, kc_stride_head;
  int64_t vc_stride_block, vc_stride_tok, vc_stride_head;
  int64_t ks_stride_block, ks_stride_tok, ks_stride_head;
  int64_t vs_stride_block, vs_stride_tok, vs_stride_head;
  int32_t num_tokens;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t block_size;
  int32_t num_blocks;
  int32_t dtype;       /* key / value: F16 / BF16 / F32 */
  int32_t cache_dtype; /* NONE: == dtype; FP8_PER_TENSOR: FP8_E4M3 / FP8_E5M2;
                          INT8_PER_TOKEN_HEAD: I8; FP8_PER_TOKEN_HEAD: FP8_E4M3 */
  int32_t quant_mode;  /* B200_KVQ_* */
  int32_t slot_dtype;  /* I32 / I64 */
} B200KvWriteParams;

B200_API int b200_kv_cache_write(const B200KvWriteParams* params, void* stream);

/*
 * Dequantise the pages a batch references, for attention over a quantised KV
 * cache (the service's fp8 / int8 caches; the reference sends those calls to
 * vLLM's unified_attention, integration/vllm-plugin-FL-split-kv.patch:473-523).
 * For sequence b and page p < ceil(seqused_k[b] / block_size), the cache rows
 * of block_table[b, p] go to dense page b * max_pages + p of out_cache
 * [num_seqs * max_pages, 2 (K, V), block_size, num_kv_heads, head_dim] in
 * out_dtype, and out_block_table[b, p] = b * max_pages + p for every p <
 * max_pages; b200_paged_attn_fwd then runs on out_cache[:, 0] / [:, 1] with
 * out_block_table.  Element values: FP8_PER_TENSOR fp8(x) * *k_scale (resp.
 * *v_scale); *_PER_TOKEN_HEAD x * scale_cache[block, slot, head]; both rounded
 * to nearest in out_dtype.  Cache element types: FP8_E4M3 / FP8_E5M2
 * (per-tensor), I8 / FP8_E4M3 (per-token-head).  Cache strides in elements
 * (bytes), multiples of 4; head_dim a multiple of 4.  A block id outside
 * [0, num_blocks) gives a zero page.
 */
typedef struct B200KvDequantParams {
  const void* key_cache;
  const void* value_cache;
  int64_t kc_stride_block, kc_stride_tok, kc_stride_head;
  int64_t vc_stride_block, vc_stride_tok, vc_stride_head;
  const float* k_scale;        /* FP8_PER_TENSOR */
  const float* v_scale;
  const float* k_scale_cache;  /* *_PER_TOKEN_HEAD, float element strides below */
  const float* v_scale_cache;
  int64_t ks_stride_block, ks_stride_tok, ks_stride_head;
  int64_t vs_stride_block, vs_stride_tok, vs_stride_head;
  const void* block_table;
  int64_t block_table_stride;
  int32_t block_table_cols;
  int32_t block_table_dtype; /* I32 / I64 */
  const void* seqused_k;
  int32_t seqlen_dtype;      /* I32 / I64 */
  void* out_cache;
  int32_t* out_block_table;  /* [num_seqs, max_pages] */
  int32_t num_seqs;
  int32_t max_pages;
  int32_t block_size;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t num_blocks;
  int32_t cache_dtype;       /* FP8_E4M3 / FP8_E5M2 / I8 */
  int32_t quant_mode;        /* B200_KVQ_FP8_PER_TENSOR / _INT8_PER_TOKEN_HEAD / _FP8_PER_TOKEN_HEAD */
  int32_t out_dtype;         /* BF16 / F16 */
} B200KvDequantParams;

B200_API int b200_kv_dequant_pages(const B200KvDequantParams* params, void* stream);

/* Message of the last failed call on this host thread ("" if none). */
B200_API const char* b200_last_error(void);

/*
 * Synchronises `stream`, then reads and clears this library's device error
 * word on the current device (B200_DEVERR_*).  For tests and debugging; the
 * hot-path calls never synchronise.
 */
B200_API int b200_device_error(void* stream, uint32_t* code);

/*
 * Test hook for the bounded waits (no reference counterpart): launches one
 * warp on `stream` that waits on an mbarrier nothing ever arrives on.  The
 * wait gives up after its limit (2 s of %globaltimer), records
 * B200_DEVERR_WAIT_TIMEOUT and the kernel returns, so the context stays
 * usable; b200_device_error then reports the timeout.  Never faults or hangs.
 */
B200_API int b200_wait_selftest(void* stream);

B200_API int b200_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MINICPM_B200_H_ */
