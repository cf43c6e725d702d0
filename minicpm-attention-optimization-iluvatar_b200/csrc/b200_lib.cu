// b200_lib.cu -- the C ABI declared in include/minicpm_b200.h.
//
// One translation unit: the kernels live in the headers included below.
// Host code validates arguments (mirroring the reference's ValueError checks
// in kernels/triton_split_kv_paged.py:249-281 and
// kernels/triton_rope_kv_cache.py:219-260 where they apply to raw pointers),
// encodes the TMA tensor maps, and enqueues the launches on the caller's
// stream.  Nothing here synchronises, allocates, or falls back to another
// implementation.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <mutex>

#include "minicpm_b200.h"
#include "paged_attention.cuh"
#include "paged_decode.cuh"
#include "rope_kv_cache.cuh"
#include "split_combine.cuh"
#include "kv_cache_write.cuh"
#include "kv_dequant.cuh"

namespace b200 {

// b200_wait_selftest: one warp waits on an mbarrier that nothing arrives on.
// The bounded wait (mbar_wait) gives up after B200_WAIT_LIMIT_NS, records
// B200_DEVERR_WAIT_TIMEOUT and raises the abort flag; the kernel then returns.
__global__ void __launch_bounds__(32, 1) wait_selftest_kernel() {
  __shared__ __align__(8) uint64_t bar_word;
  __shared__ int abort_word;
  const uint32_t bar = smem_addr(&bar_word);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    abort_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  mbar_wait(bar, 0, &abort_word);
}

}  // namespace b200

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return B200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kNumSmsB200 = 148;

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kNumSmsB200;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return kNumSmsB200;
  return n;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_map(CUtensorMap* map, CUtensorMapDataType dt, cuuint32_t rank, const void* base, const cuuint64_t* dims,
               const cuuint64_t* strides_bytes, const cuuint32_t* box, const char* what) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  const CUresult r = enc(map, dt, rank, const_cast<void*>(base), dims, strides_bytes, box, elem_strides,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200_ERR_INVALID, "tensor map for %s rejected by the driver (CUresult %d)", what, (int)r);
  return B200_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Prefill workspace: the schedule's counters and per-sequence / per-query-unit
// arrays, the work list, and (num_splits > 1) the split units' list and
// partial outputs [slot][split][256 rows][head_dim] with m / l per row.
struct WorkspaceLayout {
  size_t count_off, tile_base_off, seq_off_off, qbase_off, qsplit_off, qslot_off, units_off, split_units_off;
  size_t o_off, m_off, l_off, total;
  int capacity;
  int64_t qunits_ub, slots_ub;
};

WorkspaceLayout attn_workspace_layout(int64_t total_q, int num_seqs, int hq, int hkv, int head_dim, int splits,
                                      int elt) {
  WorkspaceLayout w{};
  const int group = hkv > 0 ? hq / hkv : 1;
  // head_dim 256: one query tile per unit, else two.
  const int ppu = std::max(group > 0 ? b200::kAttnTileM / group : 1, 1) * (head_dim == 256 ? 1 : b200::kAttnTilesPerUnit);
  w.qunits_ub = (total_q + ppu - 1) / ppu + num_seqs;
  const int64_t cap = w.qunits_ub * hkv * splits;
  w.capacity = static_cast<int>(cap > 0x7fffffff ? 0x7fffffff : cap);
  w.slots_ub = splits > 1 ? w.qunits_ub * hkv : 0;
  const size_t qn = static_cast<size_t>(w.qunits_ub);
  w.count_off = 0;
  w.tile_base_off = 256;
  w.seq_off_off = align_up(w.tile_base_off + sizeof(int) * (num_seqs + 1), 256);
  w.qbase_off = align_up(w.seq_off_off + sizeof(int) * num_seqs, 256);
  w.qsplit_off = align_up(w.qbase_off + sizeof(int) * (qn + 1), 256);
  w.qslot_off = align_up(w.qsplit_off + sizeof(int) * qn, 256);
  w.units_off = align_up(w.qslot_off + sizeof(int) * qn, 256);
  w.split_units_off = align_up(w.units_off + sizeof(int4) * static_cast<size_t>(w.capacity), 256);
  w.o_off = align_up(w.split_units_off + sizeof(int4) * static_cast<size_t>(w.slots_ub), 256);
  w.m_off = w.o_off;
  w.l_off = w.o_off;
  w.total = w.o_off;
  if (splits > 1) {
    const size_t rows = static_cast<size_t>(w.slots_ub) * splits * b200::kUnitRows;
    w.m_off = align_up(w.o_off + rows * head_dim * elt, 256);
    w.l_off = align_up(w.m_off + rows * sizeof(float), 256);
    w.total = align_up(w.l_off + rows * sizeof(float), 256);
  }
  return w;
}

// Decode batches (one query token per sequence): keys per work item, chosen so
// that the persistent grid gets about eight items per CTA.
int decode_chunk(int num_seqs, int hkv, int max_k, int num_sms) {
  const int64_t work = (int64_t)num_seqs * hkv * std::max(max_k, 1);
  const int64_t target = (int64_t)8 * std::max(num_sms, 1);
  int64_t c = (work + target - 1) / target;
  c = (c + b200::kDecTileN - 1) / b200::kDecTileN * b200::kDecTileN;
  return (int)std::min<int64_t>(std::max<int64_t>(c, 2 * b200::kDecTileN), int64_t(1) << 24);
}

struct DecodeLayout {
  size_t base_off, order_off, m_off, l_off, o_off, total;
  int chunk;
  int64_t items_ub;
};

DecodeLayout decode_layout(int num_seqs, int hkv, int group, int max_k, int num_sms) {
  DecodeLayout d{};
  d.chunk = decode_chunk(num_seqs, hkv, max_k, num_sms);
  d.items_ub = (int64_t)num_seqs * hkv * ((std::max(max_k, 0) + d.chunk - 1) / d.chunk);
  d.base_off = 0;
  d.order_off = align_up(sizeof(int) * (size_t)(num_seqs + 2), 256);
  d.m_off = align_up(d.order_off + sizeof(int) * (size_t)d.items_ub, 256);
  d.l_off = align_up(d.m_off + sizeof(float) * (size_t)d.items_ub * group, 256);
  d.o_off = align_up(d.l_off + sizeof(float) * (size_t)d.items_ub * group, 256);
  d.total = align_up(d.o_off + sizeof(float) * (size_t)d.items_ub * group * b200::kAttnHeadDim, 256);
  return d;
}

bool decode_shape_ok(int group, int hkv) {
  return (group == 4 || group == 8 || group == 16) && hkv <= b200::kDecMaxKvHeads;
}

// B200_ATTN_SPLIT_UNIFORM=1 splits every query unit num_splits ways (the
// reference's rule) instead of only the units that are a large share of the
// batch's work per SM; for measuring the split path and testing it at scale.
bool uniform_splits() {
  const char* e = getenv("B200_ATTN_SPLIT_UNIFORM");
  return e && e[0] == '1';
}

// B200_ATTN_DECODE=0 sends decode batches through the prefill kernel instead.
bool use_decode_kernel() {
  const char* e = getenv("B200_ATTN_DECODE");
  return !(e && e[0] == '0');
}

int auto_splits(int32_t total_q, int32_t num_seqs, int32_t hq, int32_t hkv, int32_t max_seqlen_k, int num_sms) {
  if (hkv <= 0 || hq <= 0 || hq % hkv) return 1;
  const int group = hq / hkv;
  const int ppt = group <= b200::kAttnTileM ? b200::kAttnTileM / group : 1;
  const int64_t units = ((int64_t)total_q + ppt - 1) / ppt * hkv;
  int s = 1;
  // Split the KV axis only while the grid is under one wave of CTAs and each
  // split keeps at least two KV tiles of work.
  while (s < b200::kMaxSplits && units * s < num_sms && (int64_t)max_seqlen_k >= (int64_t)s * 2 * 2 * b200::kAttnTileN)
    s *= 2;
  (void)num_seqs;
  return s;
}

// Decode batch: schedule (items per sequence), persistent decode kernel, combine.
// Per KV head: (d, key % 8, 64-column part of head_dim, key / 8 in the page,
// page); one box = a 16-key page slice with two parts (4 KB): the whole row at
// head_dim 128, one 128-column half of it at head_dim 256.  Needs num_kv_heads <=
// kMaxHeadMaps and block_size % 16 == 0.
int encode_kv_head_maps(const B200AttnParams* p, CUtensorMapDataType dt, b200::KvHeadMaps* maps) {
  const int elt = 2;
  memset(maps, 0, sizeof(*maps));
  for (int h = 0; h < p->num_kv_heads; ++h) {
    for (int kv = 0; kv < 2; ++kv) {
      const uint8_t* base = static_cast<const uint8_t*>(kv ? p->v : p->k) +
                            (int64_t)h * (kv ? p->v_stride_head : p->k_stride_head) * elt;
      const int64_t st = kv ? p->v_stride_tok : p->k_stride_tok, sb = kv ? p->v_stride_block : p->k_stride_block;
      const cuuint64_t dims[5] = {64, 8, (cuuint64_t)(p->head_dim / 64), (cuuint64_t)(p->block_size / 8),
                                  (cuuint64_t)p->num_blocks};
      const cuuint64_t strides[4] = {(cuuint64_t)(st * elt), 128, (cuuint64_t)(8 * st * elt), (cuuint64_t)(sb * elt)};
      const cuuint32_t box[5] = {64, 8, (cuuint32_t)std::min(2, p->head_dim / 64), 2, 1};
      if (int r = encode_map(kv ? &maps->v[h] : &maps->k[h], dt, 5, base, dims, strides, box, kv ? "v" : "k")) return r;
    }
  }
  return B200_OK;
}

int run_decode(const B200AttnParams* p, cudaStream_t s, int group) {
  const int elt = 2;
  const int sms = sm_count();
  const DecodeLayout dl = decode_layout(p->num_seqs, p->num_kv_heads, group, p->max_seqlen_k, sms);
  if (!p->workspace || p->workspace_bytes < dl.total)
    return fail(B200_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", dl.total, p->workspace_bytes);
  if (dl.items_ub == 0) return B200_OK;
  uint8_t* ws = static_cast<uint8_t*>(p->workspace);
  const CUtensorMapDataType dt =
      p->dtype == B200_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tm_q;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)p->head_dim, (cuuint64_t)p->num_q_heads, (cuuint64_t)p->total_q};
    const cuuint64_t strides[2] = {(cuuint64_t)(p->q_stride_h * elt), (cuuint64_t)(p->q_stride_t * elt)};
    const cuuint32_t box[3] = {64, (cuuint32_t)group, 1};
    if (int r = encode_map(&tm_q, dt, 3, p->q, dims, strides, box, "q")) return r;
  }
  b200::DecodeMaps maps;
  if (int r = encode_kv_head_maps(p, dt, &maps)) return r;
  b200::DecodeArgs a{};
  a.block_table = p->block_table;
  a.cu_q = p->cu_seqlens_q;
  a.seqused = p->seqused_k;
  a.item_base = reinterpret_cast<int*>(ws + dl.base_off);
  a.order = reinterpret_cast<int*>(ws + dl.order_off);
  a.part_m = reinterpret_cast<float*>(ws + dl.m_off);
  a.part_l = reinterpret_cast<float*>(ws + dl.l_off);
  a.part_o = reinterpret_cast<float*>(ws + dl.o_off);
  a.bt_stride = p->block_table_stride;
  a.bt_cols = p->block_table_cols;
  a.bt_i64 = p->block_table_dtype == B200_DTYPE_I64;
  a.len_i64 = p->seqlen_dtype == B200_DTYPE_I64;
  a.num_seqs = p->num_seqs;
  a.num_kv_heads = p->num_kv_heads;
  a.chunk = dl.chunk;
  a.block_size = p->block_size;
  a.num_blocks = p->num_blocks;
  a.scale_log2 = static_cast<float>(static_cast<double>(p->softmax_scale) * 1.4426950408889634);

  b200::decode_schedule_kernel<<<1, b200::kSchedThreads, 0, s>>>(a);
  if (int r = check_launch("decode_schedule_kernel")) return r;
  const dim3 grid((unsigned)std::min<int64_t>(sms, dl.items_ub));
  // The decode and combine kernels are launched as programmatic dependents of
  // their predecessor: each starts while the previous grid finishes and waits
  // for it (griddepcontrol.wait) before reading its output.
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  auto launch = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, b200::kDecodeSmemAlloc);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(b200::kDecThreads);
    cfg.dynamicSmemBytes = b200::kDecodeSmemAlloc;
    cfg.stream = s;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, tm_q, maps, a);
  };
  auto launch_combine = [&](auto kernel) {
    const int64_t warps = (int64_t)p->num_seqs * p->num_q_heads;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((warps + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, a, p->out, p->out_stride_t, p->out_stride_h, p->num_q_heads);
  };
#define B200_DECODE_G(T)                                                                          \
  switch (group) {                                                                                \
    case 4: launch(b200::paged_decode_kernel<T, 4>); break;                                       \
    case 8: launch(b200::paged_decode_kernel<T, 8>); break;                                       \
    default: launch(b200::paged_decode_kernel<T, 16>); break;                                     \
  }                                                                                               \
  if (int r = check_launch("paged_decode_kernel")) return r;                                      \
  switch (group) {                                                                                \
    case 4: launch_combine(b200::decode_combine_kernel<T, 4>); break;                             \
    case 8: launch_combine(b200::decode_combine_kernel<T, 8>); break;                             \
    default: launch_combine(b200::decode_combine_kernel<T, 16>); break;                           \
  }
  if (p->dtype == B200_DTYPE_BF16) {
    B200_DECODE_G(__nv_bfloat16)
  } else {
    B200_DECODE_G(__half)
  }
#undef B200_DECODE_G
  return check_launch("decode_combine_kernel");
}

}  // namespace

extern "C" {

int b200_abi_version(void) { return B200_ABI_VERSION; }

const char* b200_last_error(void) { return g_last_error; }

int32_t b200_choose_num_splits(int32_t total_q, int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                               int32_t max_seqlen_k) {
  return auto_splits(total_q, num_seqs, num_q_heads, num_kv_heads, max_seqlen_k, sm_count());
}

int32_t b200_attn_shape_supported(int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype) {
  if (dtype != B200_DTYPE_BF16 && dtype != B200_DTYPE_F16) return 0;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads) return 0;
  if (num_q_heads / num_kv_heads > b200::kAttnTileM) return 0;
  return head_dim == 64 || head_dim == b200::kAttnHeadDim || head_dim == 256;
}

size_t b200_attn_workspace_bytes(int32_t total_q, int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                                 int32_t head_dim, int32_t num_splits, int32_t max_seqlen_k, int32_t dtype) {
  if (num_splits <= 0) num_splits = b200_choose_num_splits(total_q, num_seqs, num_q_heads, num_kv_heads, max_seqlen_k);
  const int elt = (dtype == B200_DTYPE_F32) ? 4 : 2;
  size_t bytes = attn_workspace_layout(total_q, num_seqs, num_q_heads, num_kv_heads, head_dim, num_splits, elt).total;
  // A batch with at most one query token per sequence may run the decode kernel.
  if (total_q <= num_seqs && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0 && head_dim == b200::kAttnHeadDim &&
      decode_shape_ok(num_q_heads / num_kv_heads, num_kv_heads))
    bytes = std::max(bytes, decode_layout(num_seqs, num_kv_heads, num_q_heads / num_kv_heads, max_seqlen_k,
                                          sm_count()).total);
  return bytes;
}

int b200_split_combine(const B200CombineParams* p, void* stream) {
  if (!p) return fail(B200_ERR_INVALID, "null params");
  if (p->num_splits < 1 || p->num_splits > b200::kMaxSplits)
    return fail(B200_ERR_INVALID, "num_splits must be in [1, %d]", b200::kMaxSplits);
  if (p->total_q < 0 || p->num_heads <= 0) return fail(B200_ERR_INVALID, "bad sizes");
  if (p->head_dim != 64 && p->head_dim != 128 && p->head_dim != 256)
    return fail(B200_ERR_INVALID, "head_dim must be 64, 128 or 256");
  if (p->total_q == 0) return B200_OK;
  const int oe = p->o_dtype == B200_DTYPE_F32 ? 4 : 2, ue = p->out_dtype == B200_DTYPE_F32 ? 4 : 2;
  if (!aligned16(p->o_splits) || !aligned16(p->out) || ((p->o_stride_s * oe) | (p->o_stride_t * oe) | (p->o_stride_h * oe)) & 15 ||
      ((p->out_stride_t * ue) | (p->out_stride_h * ue)) & 15)
    return fail(B200_ERR_UNSUPPORTED, "split combine needs 16-byte aligned rows of O and out");
  b200::CombineArgs a{};
  a.o = p->o_splits; a.m = p->m_splits; a.l = p->l_splits; a.out = p->out;
  a.o_ss = p->o_stride_s; a.o_st = p->o_stride_t; a.o_sh = p->o_stride_h;
  a.m_ss = p->m_stride_s; a.m_st = p->m_stride_t; a.m_sh = p->m_stride_h;
  a.l_ss = p->l_stride_s; a.l_st = p->l_stride_t; a.l_sh = p->l_stride_h;
  a.out_st = p->out_stride_t; a.out_sh = p->out_stride_h;
  a.num_splits = p->num_splits; a.total_q = p->total_q; a.num_heads = p->num_heads;
  const int64_t rows = (int64_t)p->total_q * p->num_heads;
  const int rows_per_block = b200::kCombineThreads / (p->head_dim / 8);
  const dim3 grid((unsigned)((rows + rows_per_block - 1) / rows_per_block));
  cudaStream_t s = static_cast<cudaStream_t>(stream);

#define B200_COMBINE_S(TO, TOUT, D)                                                                      \
  if (p->num_splits <= 4) b200::split_combine_kernel<TO, TOUT, D, 4><<<grid, b200::kCombineThreads, 0, s>>>(a);      \
  else if (p->num_splits <= 8) b200::split_combine_kernel<TO, TOUT, D, 8><<<grid, b200::kCombineThreads, 0, s>>>(a); \
  else b200::split_combine_kernel<TO, TOUT, D, 16><<<grid, b200::kCombineThreads, 0, s>>>(a);
#define B200_COMBINE_D(TO, TOUT)                         \
  switch (p->head_dim) {                                \
    case 64: B200_COMBINE_S(TO, TOUT, 64) break;         \
    case 128: B200_COMBINE_S(TO, TOUT, 128) break;       \
    default: B200_COMBINE_S(TO, TOUT, 256) break;        \
  }
#define B200_COMBINE_OUT(TO)                                                            \
  switch (p->out_dtype) {                                                               \
    case B200_DTYPE_BF16: B200_COMBINE_D(TO, __nv_bfloat16) break;                      \
    case B200_DTYPE_F16: B200_COMBINE_D(TO, __half) break;                              \
    case B200_DTYPE_F32: B200_COMBINE_D(TO, float) break;                               \
    default: return fail(B200_ERR_INVALID, "out dtype must be f16, bf16 or f32");       \
  }
  switch (p->o_dtype) {
    case B200_DTYPE_BF16: B200_COMBINE_OUT(__nv_bfloat16) break;
    case B200_DTYPE_F16: B200_COMBINE_OUT(__half) break;
    case B200_DTYPE_F32: B200_COMBINE_OUT(float) break;
    default: return fail(B200_ERR_INVALID, "o_splits dtype must be f16, bf16 or f32");
  }
#undef B200_COMBINE_OUT
#undef B200_COMBINE_D
#undef B200_COMBINE_S
  return check_launch("split_combine_kernel");
}

int b200_paged_attn_fwd(const B200AttnParams* p, void* stream) {
  if (!p) return fail(B200_ERR_INVALID, "null params");
  if (p->dtype != B200_DTYPE_BF16 && p->dtype != B200_DTYPE_F16)
    return fail(B200_ERR_UNSUPPORTED, "q/k/v/out must be bf16 or f16 for the sm_100a kernel");
  if (p->num_q_heads <= 0 || p->num_kv_heads <= 0 || p->num_q_heads % p->num_kv_heads)
    return fail(B200_ERR_INVALID, "unsupported head shape for paged Split-KV");
  if (p->block_size <= 0 || p->block_size % 16) return fail(B200_ERR_INVALID, "unsupported head shape for paged Split-KV");
  if (p->head_dim != 64 && p->head_dim != 128 && p->head_dim != 256)
    return fail(B200_ERR_INVALID, "unsupported head shape for paged Split-KV");
  // head_dim 64 runs the kernel's narrow variant (K/V half-slots, K = 64 S
  // UMMAs, N = 64 P V UMMAs), head_dim 256 its wide variant (one query tile
  // per unit).
  const bool wide = p->head_dim == 256;
  const bool narrow = p->head_dim == 64;
  const int group = p->num_q_heads / p->num_kv_heads;
  if (group > b200::kAttnTileM)
    return fail(B200_ERR_UNSUPPORTED, "query heads per KV head (%d) must be at most 128", group);
  if (p->num_splits < 0 || p->num_splits > b200::kMaxSplits)
    return fail(B200_ERR_INVALID, "num_splits must be 0 (auto) or in [1, 16]");
  if (p->num_seqs < 0 || p->total_q < 0 || p->num_blocks <= 0 || p->block_table_cols <= 0)
    return fail(B200_ERR_INVALID, "bad sizes");
  if (p->block_table_dtype != B200_DTYPE_I32 && p->block_table_dtype != B200_DTYPE_I64)
    return fail(B200_ERR_INVALID, "block_table must contain integer physical block ids");
  if (p->seqlen_dtype != B200_DTYPE_I32 && p->seqlen_dtype != B200_DTYPE_I64)
    return fail(B200_ERR_INVALID, "cu_seqlens_q and seqused_k must be int32 or int64");
  if (p->total_q == 0 || p->num_seqs == 0) return B200_OK;
  const int elt = 2;
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out))
    return fail(B200_ERR_UNSUPPORTED, "q, k, v and out must be 16-byte aligned");
  if (((p->q_stride_t | p->q_stride_h | p->k_stride_block | p->k_stride_tok | p->k_stride_head | p->v_stride_block |
        p->v_stride_tok | p->v_stride_head | p->out_stride_t | p->out_stride_h) *
       elt) & 15)
    return fail(B200_ERR_UNSUPPORTED, "token/head/block strides must be multiples of 16 bytes");
  // Decode batches take the decode kernel (its own workspace layout and maps).
  if (p->max_seqlen_q == 1 && p->head_dim == b200::kAttnHeadDim && decode_shape_ok(group, p->num_kv_heads) &&
      use_decode_kernel())
    return run_decode(p, static_cast<cudaStream_t>(stream), group);

  const int splits = p->num_splits > 0 ? p->num_splits
                                       : b200_choose_num_splits(p->total_q, p->num_seqs, p->num_q_heads,
                                                                p->num_kv_heads, p->max_seqlen_k);
  const WorkspaceLayout w =
      attn_workspace_layout(p->total_q, p->num_seqs, p->num_q_heads, p->num_kv_heads, p->head_dim, splits, elt);
  if (!p->workspace || p->workspace_bytes < w.total)
    return fail(B200_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", w.total, p->workspace_bytes);
  if (!aligned16(p->workspace)) return fail(B200_ERR_WORKSPACE, "workspace must be 16-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(p->workspace);

  const CUtensorMapDataType dt = p->dtype == B200_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int ppt = b200::kAttnTileM / group;
  CUtensorMap tm_q, tm_k, tm_v;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)p->head_dim, (cuuint64_t)p->num_q_heads, (cuuint64_t)p->total_q};
    const cuuint64_t strides[2] = {(cuuint64_t)(p->q_stride_h * elt), (cuuint64_t)(p->q_stride_t * elt)};
    const cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)ppt};
    if (int r = encode_map(&tm_q, dt, 3, p->q, dims, strides, box, "q")) return r;
  }
  {
    const cuuint64_t dims[4] = {(cuuint64_t)p->head_dim, (cuuint64_t)p->block_size, (cuuint64_t)p->num_kv_heads,
                                (cuuint64_t)p->num_blocks};
    const cuuint32_t box[4] = {64, 16, 1, 1};
    const cuuint64_t ks[3] = {(cuuint64_t)(p->k_stride_tok * elt), (cuuint64_t)(p->k_stride_head * elt),
                              (cuuint64_t)(p->k_stride_block * elt)};
    if (int r = encode_map(&tm_k, dt, 4, p->k, dims, ks, box, "k")) return r;
    const cuuint64_t vs[3] = {(cuuint64_t)(p->v_stride_tok * elt), (cuuint64_t)(p->v_stride_head * elt),
                              (cuuint64_t)(p->v_stride_block * elt)};
    if (int r = encode_map(&tm_v, dt, 4, p->v, dims, vs, box, "v")) return r;
  }

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Per-KV-head maps (16-key page-slice boxes) when they fit.
  const bool head_maps = p->num_kv_heads <= b200::kMaxHeadMaps;
  b200::KvHeadMaps maps;
  if (head_maps) {
    if (int r = encode_kv_head_maps(p, dt, &maps)) return r;
  } else {
    memset(&maps, 0, sizeof(maps));
    maps.k[0] = tm_k;
    maps.v[0] = tm_v;
  }
  b200::SchedArgs sa{};
  sa.cu_q = p->cu_seqlens_q;
  sa.seqused = p->seqused_k;
  sa.len_i64 = p->seqlen_dtype == B200_DTYPE_I64;
  sa.num_seqs = p->num_seqs;
  sa.pos_per_unit = ppt * (wide ? 1 : b200::kAttnTilesPerUnit);
  sa.num_kv_heads = p->num_kv_heads;
  sa.num_splits = splits;
  sa.uniform_splits = uniform_splits() ? 1 : 0;
  sa.num_sms = sm_count();
  sa.capacity = w.capacity;
  sa.tile_base = reinterpret_cast<int*>(ws + w.tile_base_off);
  sa.seq_off = reinterpret_cast<int*>(ws + w.seq_off_off);
  sa.qunit_base = reinterpret_cast<int*>(ws + w.qbase_off);
  sa.qunit_split = reinterpret_cast<int*>(ws + w.qsplit_off);
  sa.qunit_slot = reinterpret_cast<int*>(ws + w.qslot_off);
  sa.units = reinterpret_cast<int4*>(ws + w.units_off);
  sa.split_units = reinterpret_cast<int4*>(ws + w.split_units_off);
  sa.unit_count = reinterpret_cast<int*>(ws + w.count_off);
  cudaFuncSetAttribute(b200::attn_schedule_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, b200::kSchedSmemBytes);
  b200::attn_schedule_kernel<<<1, b200::kSchedThreads, b200::kSchedSmemBytes, s>>>(sa);
  if (int r = check_launch("attn_schedule_kernel")) return r;

  b200::AttnKernelArgs a{};
  a.block_table = p->block_table;
  a.cu_q = p->cu_seqlens_q;
  a.seqused = p->seqused_k;
  a.out = p->out;
  a.o_split = ws + w.o_off;
  a.m_split = reinterpret_cast<float*>(ws + w.m_off);
  a.l_split = reinterpret_cast<float*>(ws + w.l_off);
  a.units = sa.units;
  a.unit_count = sa.unit_count;
  a.bt_stride = p->block_table_stride;
  a.out_st = p->out_stride_t;
  a.out_sh = p->out_stride_h;
  a.bt_cols = p->block_table_cols;
  a.bt_i64 = p->block_table_dtype == B200_DTYPE_I64;
  a.len_i64 = sa.len_i64;
  a.total_q = p->total_q;
  a.num_q_heads = p->num_q_heads;
  a.group = group;
  a.pos_per_tile = ppt;
  a.block_size = p->block_size;
  a.num_blocks = p->num_blocks;
  a.num_splits = splits;
  a.head_dim = p->head_dim;
  a.scale_log2 = static_cast<float>(static_cast<double>(p->softmax_scale) * 1.4426950408889634);

  // Upper bound on work units; the kernel is persistent: one CTA per SM at most.
  const int64_t units_ub =
      ((int64_t)p->total_q + sa.pos_per_unit - 1) / sa.pos_per_unit + p->num_seqs;
  const int64_t ctas = units_ub * p->num_kv_heads * splits;
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(ctas, sm_count())));
  auto launch = [&](auto kernel, const auto&... args) -> int {
    // The kernel rebalances registers between warpgroups with setmaxnreg; the
    // split adds up only if every thread was launched with exactly
    // kAttnLaunchRegs registers, so refuse to launch otherwise.
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess || fa.numRegs != b200::kAttnLaunchRegs)
      return fail(B200_ERR_CUDA, "paged_attn_fwd_kernel built with %d registers per thread, %d expected", fa.numRegs,
                  b200::kAttnLaunchRegs);
    const uint32_t smem = b200::kAttnSmemAlloc;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    // A programmatic dependent of the schedule kernel: launched while it runs,
    // it waits for it (griddepcontrol.wait) before reading the work list.
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(b200::kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, args...);
    return B200_OK;
  };
  const bool bf16 = p->dtype == B200_DTYPE_BF16;
  int lr;
#define B200_ATTN_LAUNCH(HM, WIDE, NARROW)                                                           \
  lr = bf16 ? launch(b200::paged_attn_fwd_kernel<__nv_bfloat16, HM, WIDE, NARROW>, tm_q, maps, a)    \
            : launch(b200::paged_attn_fwd_kernel<__half, HM, WIDE, NARROW>, tm_q, maps, a);
#define B200_ATTN_MAPS(WIDE, NARROW) \
  if (head_maps) { B200_ATTN_LAUNCH(true, WIDE, NARROW) } else { B200_ATTN_LAUNCH(false, WIDE, NARROW) }
  if (wide) {
    B200_ATTN_MAPS(true, false)
  } else if (narrow) {
    B200_ATTN_MAPS(false, true)
  } else {
    B200_ATTN_MAPS(false, false)
  }
#undef B200_ATTN_MAPS
#undef B200_ATTN_LAUNCH
  if (lr != B200_OK) return lr;
  if (int r = check_launch("paged_attn_fwd_kernel")) return r;

  if (splits > 1) {
    // Combine of the split units' partials; the split-unit count is on the
    // device, so the grid is a bound and the kernel loops up to the count.
    b200::UnitCombineArgs c{};
    c.o_part = a.o_split;
    c.m_part = a.m_split;
    c.l_part = a.l_split;
    c.split_units = sa.split_units;
    c.unit_count = sa.unit_count;
    c.cu_q = p->cu_seqlens_q;
    c.out = p->out;
    c.out_st = p->out_stride_t;
    c.out_sh = p->out_stride_h;
    c.len_i64 = sa.len_i64;
    c.num_splits = splits;
    c.group = group;
    c.pos_per_tile = ppt;
    c.pos_per_unit = sa.pos_per_unit;
    const int rows_per_block = b200::kCombineThreads / (p->head_dim / 8);
    const int64_t blocks_ub = (w.slots_ub * b200::kUnitRows + rows_per_block - 1) / rows_per_block;
    // Eight CTAs per SM at most (grid-stride over the split rows: enough rows
    // in flight to stream the partials at HBM speed); launched as a
    // programmatic dependent of the attention kernel, so a call whose units
    // were not split pays little more than the launch.
    cudaLaunchAttribute cpdl[1];
    cpdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    cpdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t ccfg{};
    ccfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks_ub, (int64_t)sm_count() * 8)));
    ccfg.blockDim = dim3(b200::kCombineThreads);
    ccfg.stream = s;
    ccfg.attrs = cpdl;
    ccfg.numAttrs = 1;
#define B200_UCOMB_S(T, D)                                                                     \
  if (splits <= 4) cudaLaunchKernelEx(&ccfg, b200::unit_combine_kernel<T, D, 4>, c);          \
  else if (splits <= 8) cudaLaunchKernelEx(&ccfg, b200::unit_combine_kernel<T, D, 8>, c);     \
  else cudaLaunchKernelEx(&ccfg, b200::unit_combine_kernel<T, D, 16>, c);
#define B200_UCOMB_D(T)                                                                          \
  if (p->head_dim == 64) { B200_UCOMB_S(T, 64) } else if (p->head_dim == 128) { B200_UCOMB_S(T, 128) } \
  else { B200_UCOMB_S(T, 256) }
    if (bf16) { B200_UCOMB_D(__nv_bfloat16) } else { B200_UCOMB_D(__half) }
#undef B200_UCOMB_D
#undef B200_UCOMB_S
    return check_launch("unit_combine_kernel");
  }
  return B200_OK;
}

int b200_rope_kv_write(const B200RopeParams* p, void* stream) {
  if (!p) return fail(B200_ERR_INVALID, "null params");
  if (p->dtype != B200_DTYPE_BF16 && p->dtype != B200_DTYPE_F16)
    return fail(B200_ERR_INVALID, "only unquantized BF16/FP16 caches are supported");
  if (p->position_dtype != B200_DTYPE_I32 && p->position_dtype != B200_DTYPE_I64)
    return fail(B200_ERR_INVALID, "positions and slot_mapping must contain integer indices");
  if (p->slot_dtype != B200_DTYPE_I32 && p->slot_dtype != B200_DTYPE_I64)
    return fail(B200_ERR_INVALID, "positions and slot_mapping must contain integer indices");
  if (p->cos_sin_dtype != B200_DTYPE_BF16 && p->cos_sin_dtype != B200_DTYPE_F16 && p->cos_sin_dtype != B200_DTYPE_F32)
    return fail(B200_ERR_INVALID, "cos_sin_cache must be f16, bf16 or f32");
  if (p->rotary_dim <= 0 || p->rotary_dim > p->head_dim || p->rotary_dim % 2 || p->num_q_heads < p->num_kv_heads ||
      (p->head_dim != 64 && p->head_dim != 128 && p->head_dim != 256) || p->block_size <= 0 || p->block_size % 16 ||
      p->num_kv_heads <= 0)
    return fail(B200_ERR_INVALID, "unsupported RoPE/cache shape");
  const bool fp8_cache = p->cache_dtype == B200_DTYPE_FP8_E4M3 || p->cache_dtype == B200_DTYPE_FP8_E5M2;
  if (p->cache_dtype != p->dtype && !fp8_cache)
    return fail(B200_ERR_INVALID, "the caches must have the query dtype or be float8 e4m3 / e5m2");
  if (fp8_cache && (!p->k_scale || !p->v_scale)) return fail(B200_ERR_INVALID, "fp8 caches need k_scale and v_scale");
  const bool svc = fp8_cache || p->key_out != nullptr;
  if (p->num_tokens <= 0) return B200_OK;

  b200::RopeArgs a{};
  a.q = p->query; a.k = p->key; a.v = p->value; a.pos = p->positions; a.cs = p->cos_sin_cache;
  a.kc = p->key_cache; a.vc = p->value_cache; a.slot = p->slot_mapping;
  a.q_st = p->q_stride_t; a.q_sh = p->q_stride_h; a.q_sd = p->q_stride_d;
  a.k_st = p->k_stride_t; a.k_sh = p->k_stride_h; a.k_sd = p->k_stride_d;
  a.v_st = p->v_stride_t; a.v_sh = p->v_stride_h; a.v_sd = p->v_stride_d;
  a.cs_st = p->cos_sin_stride_t;
  a.c_sb = p->cache_stride_block; a.c_st = p->cache_stride_tok; a.c_sh = p->cache_stride_head; a.c_sd = p->cache_stride_d;
  a.num_slots = (int64_t)p->num_blocks * p->block_size;
  a.num_tokens = p->num_tokens; a.hq = p->num_q_heads; a.hkv = p->num_kv_heads; a.head_dim = p->head_dim;
  a.rd = p->rotary_dim; a.block_size = p->block_size; a.max_position = p->max_position;
  a.pos_i64 = p->position_dtype == B200_DTYPE_I64;
  a.slot_i64 = p->slot_dtype == B200_DTYPE_I64;
  a.ko = p->key_out; a.ko_st = p->ko_stride_t; a.ko_sh = p->ko_stride_h;
  a.cache_elem = p->cache_dtype == B200_DTYPE_FP8_E4M3 ? b200::kElemE4M3
                 : p->cache_dtype == B200_DTYPE_FP8_E5M2 ? b200::kElemE5M2 : b200::kElemSame;
  a.k_scale = p->k_scale; a.v_scale = p->v_scale;

  const int cse = p->cos_sin_dtype == B200_DTYPE_F32 ? 4 : 2;
  // Cache rows: 16-byte aligned for the model dtype, 4-byte for fp8.
  const int64_t ce = fp8_cache ? 1 : 2, calign = fp8_cache ? 4 : 16;
  const bool cache_ok = p->cache_stride_d == 1 &&
                        (reinterpret_cast<uintptr_t>(p->key_cache) | reinterpret_cast<uintptr_t>(p->value_cache)) %
                                calign == 0 &&
                        ((p->cache_stride_block | p->cache_stride_tok | p->cache_stride_head) * ce) % calign == 0;
  const bool vec_ok = p->q_stride_d == 1 && p->k_stride_d == 1 && p->v_stride_d == 1 && cache_ok &&
                      aligned16(p->query) && aligned16(p->key) && aligned16(p->value) && aligned16(p->cos_sin_cache) &&
                      (((p->q_stride_t | p->q_stride_h | p->k_stride_t | p->k_stride_h | p->v_stride_t | p->v_stride_h) *
                        2) & 15) == 0 &&
                      ((p->cos_sin_stride_t * cse) & 15) == 0 &&
                      (!p->key_out || (aligned16(p->key_out) && (((p->ko_stride_t | p->ko_stride_h) * 2) & 15) == 0)) &&
                      (p->is_neox ? (p->rotary_dim % 16 == 0) : (p->rotary_dim % 8 == 0));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nc = p->is_neox ? p->rotary_dim / 16 : p->rotary_dim / 8;  // rotation units per head
  const bool warp_ok = vec_ok && (nc == 4 || nc == 8 || nc == 16);
  if (svc && !warp_ok)
    return fail(B200_ERR_UNSUPPORTED,
                "key_out / fp8 caches need 16-byte aligned rows with contiguous head_dim and rotary_dim "
                "64, 128 or 256 (NeoX) or 32, 64 or 128 (interleaved)");
  if (warp_ok) {
    // Warp per token, grid-stride: exactly the CTAs that fit on the GPU at
    // once (no partial second wave), or fewer when there are few tokens.
    const int64_t warps_per_cta = b200::kRopeThreads / 32;
    auto launch = [&](auto kernel) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, b200::kRopeThreads, 0) != cudaSuccess || per_sm <= 0)
        per_sm = 1;
      const int64_t resident = (int64_t)sm_count() * per_sm;
      const int64_t needed = (p->num_tokens + warps_per_cta - 1) / warps_per_cta;
      const dim3 grid((unsigned)std::max<int64_t>(1, std::min(resident, needed)));
      kernel<<<grid, b200::kRopeThreads, 0, s>>>(a);
    };
#define B200_ROPE_WARP_SVC(T, CS, NEOX, NC)                                        \
  if (svc) launch(b200::rope_kv_warp_kernel<T, CS, NEOX, NC, true>);               \
  else launch(b200::rope_kv_warp_kernel<T, CS, NEOX, NC, false>);
#define B200_ROPE_WARP_NC(T, CS, NEOX)                                       \
  switch (nc) {                                                              \
    case 4: B200_ROPE_WARP_SVC(T, CS, NEOX, 4) break;                        \
    case 8: B200_ROPE_WARP_SVC(T, CS, NEOX, 8) break;                        \
    default: B200_ROPE_WARP_SVC(T, CS, NEOX, 16) break;                      \
  }
#define B200_ROPE_WARP(T, CS)                   \
  if (p->is_neox) { B200_ROPE_WARP_NC(T, CS, true) } else { B200_ROPE_WARP_NC(T, CS, false) }
#define B200_ROPE_WARP_CS(T)                                                  \
  switch (p->cos_sin_dtype) {                                                 \
    case B200_DTYPE_BF16: B200_ROPE_WARP(T, __nv_bfloat16) break;             \
    case B200_DTYPE_F16: B200_ROPE_WARP(T, __half) break;                     \
    default: B200_ROPE_WARP(T, float) break;                                  \
  }
    if (p->dtype == B200_DTYPE_BF16) { B200_ROPE_WARP_CS(__nv_bfloat16) } else { B200_ROPE_WARP_CS(__half) }
#undef B200_ROPE_WARP_CS
#undef B200_ROPE_WARP
#undef B200_ROPE_WARP_NC
#undef B200_ROPE_WARP_SVC
    return check_launch("rope_kv_warp_kernel");
  }
  if (vec_ok) {
    const int half = p->rotary_dim / 2;
    const int n_rot = p->is_neox ? half / 8 : p->rotary_dim / 8;
    const int per_token = p->num_q_heads * n_rot + p->num_kv_heads * (n_rot + (p->head_dim - p->rotary_dim) / 8) +
                          p->num_kv_heads * (p->head_dim / 8);
    const int64_t threads = (int64_t)per_token * p->num_tokens;
    const dim3 grid((unsigned)((threads + b200::kRopeThreads - 1) / b200::kRopeThreads));
#define B200_ROPE_VEC(T, CS)                                                                                     \
  if (p->is_neox) b200::rope_kv_vec_kernel<T, CS, true><<<grid, b200::kRopeThreads, 0, s>>>(a);                   \
  else b200::rope_kv_vec_kernel<T, CS, false><<<grid, b200::kRopeThreads, 0, s>>>(a);
#define B200_ROPE_CS(T)                                                         \
  switch (p->cos_sin_dtype) {                                                   \
    case B200_DTYPE_BF16: B200_ROPE_VEC(T, __nv_bfloat16) break;                \
    case B200_DTYPE_F16: B200_ROPE_VEC(T, __half) break;                        \
    default: B200_ROPE_VEC(T, float) break;                                     \
  }
    if (p->dtype == B200_DTYPE_BF16) { B200_ROPE_CS(__nv_bfloat16) } else { B200_ROPE_CS(__half) }
#undef B200_ROPE_CS
#undef B200_ROPE_VEC
    return check_launch("rope_kv_vec_kernel");
  }
  const int half = p->rotary_dim / 2;
  const int per_token = p->num_q_heads * half + p->num_kv_heads * (half + (p->head_dim - p->rotary_dim)) +
                        p->num_kv_heads * p->head_dim;
  const int64_t threads = (int64_t)per_token * p->num_tokens;
  const dim3 grid((unsigned)((threads + b200::kRopeThreads - 1) / b200::kRopeThreads));
#define B200_ROPE_SC(T, CS) b200::rope_kv_scalar_kernel<T, CS><<<grid, b200::kRopeThreads, 0, s>>>(a, p->is_neox);
#define B200_ROPE_SCS(T)                                                 \
  switch (p->cos_sin_dtype) {                                            \
    case B200_DTYPE_BF16: B200_ROPE_SC(T, __nv_bfloat16) break;          \
    case B200_DTYPE_F16: B200_ROPE_SC(T, __half) break;                  \
    default: B200_ROPE_SC(T, float) break;                               \
  }
  if (p->dtype == B200_DTYPE_BF16) { B200_ROPE_SCS(__nv_bfloat16) } else { B200_ROPE_SCS(__half) }
#undef B200_ROPE_SCS
#undef B200_ROPE_SC
  return check_launch("rope_kv_scalar_kernel");
}

int b200_kv_cache_write(const B200KvWriteParams* p, void* stream) {
  if (!p) return fail(B200_ERR_INVALID, "null params");
  if (p->dtype != B200_DTYPE_BF16 && p->dtype != B200_DTYPE_F16 && p->dtype != B200_DTYPE_F32)
    return fail(B200_ERR_INVALID, "key/value must be f16, bf16 or f32");
  if (p->slot_dtype != B200_DTYPE_I32 && p->slot_dtype != B200_DTYPE_I64)
    return fail(B200_ERR_INVALID, "slot_mapping must contain int32 or int64 indices");
  if ((p->head_dim != 64 && p->head_dim != 128 && p->head_dim != 256) || p->num_kv_heads <= 0 || p->block_size <= 0 ||
      p->num_blocks < 0)
    return fail(B200_ERR_INVALID, "unsupported KV-cache shape (head_dim must be 64, 128 or 256)");
  int elem = b200::kElemSame;
  switch (p->quant_mode) {
    case B200_KVQ_NONE:
      if (p->cache_dtype != p->dtype) return fail(B200_ERR_INVALID, "an unquantised cache must have the key dtype");
      break;
    case B200_KVQ_FP8_PER_TENSOR:
      if (p->cache_dtype != B200_DTYPE_FP8_E4M3 && p->cache_dtype != B200_DTYPE_FP8_E5M2)
        return fail(B200_ERR_INVALID, "fp8 per-tensor caches must be float8 e4m3 or e5m2");
      if (!p->k_scale || !p->v_scale) return fail(B200_ERR_INVALID, "fp8 per-tensor caches need k_scale and v_scale");
      elem = p->cache_dtype == B200_DTYPE_FP8_E4M3 ? b200::kElemE4M3 : b200::kElemE5M2;
      break;
    case B200_KVQ_INT8_PER_TOKEN_HEAD:
    case B200_KVQ_FP8_PER_TOKEN_HEAD: {
      const int want = p->quant_mode == B200_KVQ_INT8_PER_TOKEN_HEAD ? B200_DTYPE_I8 : B200_DTYPE_FP8_E4M3;
      if (p->cache_dtype != want)
        return fail(B200_ERR_INVALID, "per-token-head caches must be int8 (int8 mode) or float8 e4m3 (fp8 mode)");
      if (!p->k_scale_cache || !p->v_scale_cache)
        return fail(B200_ERR_INVALID, "per-token-head caches need k_scale_cache and v_scale_cache");
      elem = p->quant_mode == B200_KVQ_INT8_PER_TOKEN_HEAD ? b200::kElemI8 : b200::kElemE4M3;
      break;
    }
    default:
      return fail(B200_ERR_UNSUPPORTED, "KV quantisation mode %d is not supported", p->quant_mode);
  }
  if (p->num_tokens <= 0) return B200_OK;
  const int64_t ie = p->dtype == B200_DTYPE_F32 ? 4 : 2;
  if (!aligned16(p->key) || !aligned16(p->value) ||
      ((p->k_stride_t | p->k_stride_h | p->v_stride_t | p->v_stride_h) * ie) & 15)
    return fail(B200_ERR_UNSUPPORTED, "key/value rows must be 16-byte aligned with contiguous head_dim");
  const int64_t ce = p->quant_mode == B200_KVQ_NONE ? ie : 1;
  const int64_t calign = p->quant_mode == B200_KVQ_NONE ? 16 : 4;
  if ((reinterpret_cast<uintptr_t>(p->key_cache) | reinterpret_cast<uintptr_t>(p->value_cache)) % calign ||
      ((p->kc_stride_block | p->kc_stride_tok | p->kc_stride_head | p->vc_stride_block | p->vc_stride_tok |
        p->vc_stride_head) * ce) % calign)
    return fail(B200_ERR_UNSUPPORTED, "cache rows must be %d-byte aligned with contiguous head_dim", (int)calign);

  b200::KvWriteArgs a{};
  a.k = p->key; a.v = p->value; a.kc = p->key_cache; a.vc = p->value_cache; a.slot = p->slot_mapping;
  a.k_scale = p->k_scale; a.v_scale = p->v_scale; a.ksc = p->k_scale_cache; a.vsc = p->v_scale_cache;
  a.k_st = p->k_stride_t; a.k_sh = p->k_stride_h; a.v_st = p->v_stride_t; a.v_sh = p->v_stride_h;
  a.kc_sb = p->kc_stride_block; a.kc_st = p->kc_stride_tok; a.kc_sh = p->kc_stride_head;
  a.vc_sb = p->vc_stride_block; a.vc_st = p->vc_stride_tok; a.vc_sh = p->vc_stride_head;
  a.ks_sb = p->ks_stride_block; a.ks_st = p->ks_stride_tok; a.ks_sh = p->ks_stride_head;
  a.vs_sb = p->vs_stride_block; a.vs_st = p->vs_stride_tok; a.vs_sh = p->vs_stride_head;
  a.num_slots = (int64_t)p->num_blocks * p->block_size;
  a.num_tokens = p->num_tokens; a.hkv = p->num_kv_heads; a.head_dim = p->head_dim; a.block_size = p->block_size;
  a.slot_i64 = p->slot_dtype == B200_DTYPE_I64;
  const int64_t n_items = (int64_t)p->num_tokens * p->num_kv_heads * (p->head_dim / 8);
  if (n_items >= (int64_t(1) << 31) || a.num_slots >= (int64_t(1) << 31))
    return fail(B200_ERR_UNSUPPORTED, "more than 2^31 chunks or cache slots in one KV-cache write");
  auto log2_or = [](int64_t v) {
    if (v <= 0 || (v & (v - 1))) return -1;
    int k = 0;
    while ((int64_t(1) << k) < v) ++k;
    return k;
  };
  a.total_items = (uint32_t)n_items;
  a.n_shift = log2_or((int64_t)p->num_kv_heads * (p->head_dim / 8));
  a.bs_shift = log2_or(p->block_size);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kernel) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, b200::kKvWriteThreads, 0) != cudaSuccess ||
        per_sm <= 0)
      per_sm = 1;
    const int64_t resident = (int64_t)sm_count() * per_sm;
    const int64_t needed = (n_items + b200::kKvWriteThreads - 1) / b200::kKvWriteThreads;
    kernel<<<dim3((unsigned)std::max<int64_t>(1, std::min(resident, needed))), b200::kKvWriteThreads, 0, s>>>(a);
  };
#define B200_KV_CPR(T, MODE, ELEM)                                              \
  switch (p->head_dim) {                                                        \
    case 64: launch(b200::kv_cache_write_kernel<T, MODE, ELEM, 8>); break;      \
    case 128: launch(b200::kv_cache_write_kernel<T, MODE, ELEM, 16>); break;    \
    default: launch(b200::kv_cache_write_kernel<T, MODE, ELEM, 32>); break;     \
  }
#define B200_KV_MODES(T)                                                                      \
  if (p->quant_mode == B200_KVQ_NONE) { B200_KV_CPR(T, b200::kKvCopy, b200::kElemSame) }      \
  else if (p->quant_mode == B200_KVQ_FP8_PER_TENSOR) {                                        \
    if (elem == b200::kElemE4M3) { B200_KV_CPR(T, b200::kKvFp8Tensor, b200::kElemE4M3) }      \
    else { B200_KV_CPR(T, b200::kKvFp8Tensor, b200::kElemE5M2) }                              \
  } else if (elem == b200::kElemI8) { B200_KV_CPR(T, b200::kKvPerTokenHead, b200::kElemI8) }  \
  else { B200_KV_CPR(T, b200::kKvPerTokenHead, b200::kElemE4M3) }
  switch (p->dtype) {
    case B200_DTYPE_BF16: B200_KV_MODES(__nv_bfloat16) break;
    case B200_DTYPE_F16: B200_KV_MODES(__half) break;
    default: B200_KV_MODES(float) break;
  }
#undef B200_KV_MODES
#undef B200_KV_CPR
  return check_launch("kv_cache_write_kernel");
}

int b200_kv_dequant_pages(const B200KvDequantParams* p, void* stream) {
  if (!p) return fail(B200_ERR_INVALID, "null params");
  const bool per_tensor = p->quant_mode == B200_KVQ_FP8_PER_TENSOR;
  const bool per_token_head =
      p->quant_mode == B200_KVQ_INT8_PER_TOKEN_HEAD || p->quant_mode == B200_KVQ_FP8_PER_TOKEN_HEAD;
  if (!per_tensor && !per_token_head)
    return fail(B200_ERR_UNSUPPORTED, "KV quantisation mode %d has no dequantisation here", p->quant_mode);
  if (per_tensor && p->cache_dtype != B200_DTYPE_FP8_E4M3 && p->cache_dtype != B200_DTYPE_FP8_E5M2)
    return fail(B200_ERR_INVALID, "fp8 per-tensor caches must be float8 e4m3 or e5m2");
  if (p->quant_mode == B200_KVQ_INT8_PER_TOKEN_HEAD && p->cache_dtype != B200_DTYPE_I8)
    return fail(B200_ERR_INVALID, "int8 per-token-head caches must be int8");
  if (p->quant_mode == B200_KVQ_FP8_PER_TOKEN_HEAD && p->cache_dtype != B200_DTYPE_FP8_E4M3)
    return fail(B200_ERR_INVALID, "fp8 per-token-head caches must be float8 e4m3");
  if (per_tensor && (!p->k_scale || !p->v_scale)) return fail(B200_ERR_INVALID, "fp8 per-tensor caches need k_scale and v_scale");
  if (per_token_head && (!p->k_scale_cache || !p->v_scale_cache))
    return fail(B200_ERR_INVALID, "per-token-head caches need k_scale_cache and v_scale_cache");
  if (p->out_dtype != B200_DTYPE_BF16 && p->out_dtype != B200_DTYPE_F16)
    return fail(B200_ERR_INVALID, "the dequantised cache must be bf16 or f16");
  if (p->block_table_dtype != B200_DTYPE_I32 && p->block_table_dtype != B200_DTYPE_I64)
    return fail(B200_ERR_INVALID, "block_table must contain integer physical block ids");
  if (p->seqlen_dtype != B200_DTYPE_I32 && p->seqlen_dtype != B200_DTYPE_I64)
    return fail(B200_ERR_INVALID, "seqused_k must be int32 or int64");
  if (p->num_seqs < 0 || p->max_pages < 0 || p->block_size <= 0 || p->num_kv_heads <= 0 || p->head_dim <= 0 ||
      p->head_dim % 4 || p->num_blocks < 0)
    return fail(B200_ERR_INVALID, "bad sizes");
  if (((reinterpret_cast<uintptr_t>(p->key_cache) | reinterpret_cast<uintptr_t>(p->value_cache)) & 3) ||
      ((p->kc_stride_block | p->kc_stride_tok | p->kc_stride_head | p->vc_stride_block | p->vc_stride_tok |
        p->vc_stride_head) & 3))
    return fail(B200_ERR_UNSUPPORTED, "cache rows must be 4-byte aligned");
  if (!aligned16(p->out_cache)) return fail(B200_ERR_INVALID, "out_cache must be 16-byte aligned");
  if (p->num_seqs == 0 || p->max_pages == 0) return B200_OK;
  if ((int64_t)p->max_pages * p->num_seqs >= (int64_t(1) << 31) || p->num_seqs > 65535)
    return fail(B200_ERR_UNSUPPORTED, "too many pages or sequences for one dequantisation launch");
  b200::KvDequantArgs a{};
  a.kc = static_cast<const uint8_t*>(p->key_cache);
  a.vc = static_cast<const uint8_t*>(p->value_cache);
  a.kc_sb = p->kc_stride_block; a.kc_st = p->kc_stride_tok; a.kc_sh = p->kc_stride_head;
  a.vc_sb = p->vc_stride_block; a.vc_st = p->vc_stride_tok; a.vc_sh = p->vc_stride_head;
  a.k_scale = p->k_scale; a.v_scale = p->v_scale; a.ksc = p->k_scale_cache; a.vsc = p->v_scale_cache;
  a.ks_sb = p->ks_stride_block; a.ks_st = p->ks_stride_tok; a.ks_sh = p->ks_stride_head;
  a.vs_sb = p->vs_stride_block; a.vs_st = p->vs_stride_tok; a.vs_sh = p->vs_stride_head;
  a.block_table = p->block_table; a.bt_stride = p->block_table_stride; a.bt_cols = p->block_table_cols;
  a.bt_i64 = p->block_table_dtype == B200_DTYPE_I64;
  a.seqused = p->seqused_k; a.len_i64 = p->seqlen_dtype == B200_DTYPE_I64;
  a.out = p->out_cache; a.out_table = p->out_block_table;
  a.num_seqs = p->num_seqs; a.max_pages = p->max_pages; a.block_size = p->block_size; a.hkv = p->num_kv_heads;
  a.head_dim = p->head_dim; a.num_blocks = p->num_blocks;
  const int64_t pages = (int64_t)p->max_pages * p->num_seqs;
  const dim3 grid((unsigned)std::max<int64_t>(1, std::min<int64_t>(pages, (int64_t)sm_count() * 8)));
  const bool vec8 = p->head_dim % 8 == 0 &&
                    ((reinterpret_cast<uintptr_t>(p->key_cache) | reinterpret_cast<uintptr_t>(p->value_cache)) & 7) == 0 &&
                    ((p->kc_stride_block | p->kc_stride_tok | p->kc_stride_head | p->vc_stride_block |
                      p->vc_stride_tok | p->vc_stride_head) & 7) == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define B200_DQ(T, ELEM, PTH)                                                                         \
  if (vec8) b200::kv_dequant_kernel<T, ELEM, PTH, 8><<<grid, b200::kDequantThreads, 0, s>>>(a);       \
  else b200::kv_dequant_kernel<T, ELEM, PTH, 4><<<grid, b200::kDequantThreads, 0, s>>>(a);
#define B200_DQ_T(T)                                                                               \
  if (p->quant_mode == B200_KVQ_FP8_PER_TENSOR) {                                                  \
    if (p->cache_dtype == B200_DTYPE_FP8_E4M3) { B200_DQ(T, b200::kElemE4M3, false) }             \
    else { B200_DQ(T, b200::kElemE5M2, false) }                                                    \
  } else if (p->quant_mode == B200_KVQ_INT8_PER_TOKEN_HEAD) { B200_DQ(T, b200::kElemI8, true) }   \
  else { B200_DQ(T, b200::kElemE4M3, true) }
  if (p->out_dtype == B200_DTYPE_BF16) { B200_DQ_T(__nv_bfloat16) } else { B200_DQ_T(__half) }
#undef B200_DQ_T
#undef B200_DQ
  return check_launch("kv_dequant_kernel");
}

int b200_wait_selftest(void* stream) {
  b200::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  return check_launch("wait_selftest_kernel");
}

int b200_device_error(void* stream, uint32_t* code) {
  if (!code) return fail(B200_ERR_INVALID, "null code pointer");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "stream synchronize: %s", cudaGetErrorString(e));
  unsigned int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, b200::g_device_error, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(b200::g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "device error word: %s", cudaGetErrorString(e));
  *code = v;
  return B200_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of b200_paged_attn_fwd.
//
// Some callers cannot hand this library a workspace: a serving engine that
// reserved nearly all of HBM for its KV-cache pages at start-up and forbids
// later allocations, a host runtime in another language that reaches this
// code through the C ABI and has no device allocator of its own, or a caller
// on a latency-critical path where cudaMalloc/cudaFree would synchronise the
// device.  For them the scratch (work list, per-sequence tile offsets and,
// when the KV axis is split, the partial outputs and their m/l statistics)
// lives in one file-scope device array of B200_STATIC_SCRATCH_BYTES, which
// every GPU that loads this library holds until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = B200_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_scratch_mu;
void* g_static_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" {

int b200_paged_attn_fwd_noalloc(const B200AttnParams* p, void* stream) {
  if (!p) return fail(B200_ERR_INVALID, "null params");
  // Size check first: pure host arithmetic, identical to the workspace query.
  const size_t need = b200_attn_workspace_bytes(p->total_q, p->num_seqs, p->num_q_heads, p->num_kv_heads,
                                                p->head_dim, p->num_splits, p->max_seqlen_k, p->dtype);
  if (need > kStaticScratchBytes)
    return fail(B200_ERR_INVALID,
                "b200_paged_attn_fwd_noalloc: this call needs %zu bytes of scratch but the static scratch holds "
                "%zu; use b200_paged_attn_fwd with a caller-owned workspace (or fewer splits)",
                need, kStaticScratchBytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(B200_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(B200_ERR_UNSUPPORTED, "device index %d out of range", dev);
  void* scratch = nullptr;
  {
    // Set-up, once per device, with that device current: the host-side name
    // g_static_scratch is only a stand-in, the kernel needs the device address.
    // The address is kept for the life of the process (the header tells
    // callers not to use this entry point across a device reset).
    std::lock_guard<std::mutex> lock(g_static_scratch_mu);
    if (!g_static_scratch_ptr[dev]) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_static_scratch);
      if (e != cudaSuccess || !ptr)
        return fail(B200_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
      g_static_scratch_ptr[dev] = ptr;
    }
    scratch = g_static_scratch_ptr[dev];
  }
  B200AttnParams q = *p;
  q.workspace = scratch;
  q.workspace_bytes = kStaticScratchBytes;
  return b200_paged_attn_fwd(&q, stream);
}

}  // extern "C"
