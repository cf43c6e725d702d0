"""ctypes binding of the C ABI in ``include/minicpm_b200.h``.

The shared library is built in place by ``build.py`` into
``minicpm_b200/_lib/libminicpm_b200.so``.  There is no fallback: if the
library is missing, every operator raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libminicpm_b200.so"

B200_OK = 0
B200_ERR_INVALID = 1
B200_ERR_UNSUPPORTED = 2
B200_ERR_CUDA = 3
B200_ERR_WORKSPACE = 4

DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2
DTYPE_I32 = 3
DTYPE_I64 = 4
DTYPE_FP8_E4M3 = 5
DTYPE_FP8_E5M2 = 6
DTYPE_I8 = 7

# KV-cache quantisation modes (numbering of vLLM's KVQuantMode).
KVQ_NONE = 0
KVQ_FP8_PER_TENSOR = 1
KVQ_INT8_PER_TOKEN_HEAD = 2
KVQ_FP8_PER_TOKEN_HEAD = 3

ABI_VERSION = 2

DEVERR_NONE = 0
DEVERR_WAIT_TIMEOUT = 1
DEVERR_SLOT_RANGE = 2
DEVERR_POS_RANGE = 3
DEVERR_DECODE_QLEN = 4

_TORCH_DTYPES = {
    torch.float16: DTYPE_F16,
    torch.bfloat16: DTYPE_BF16,
    torch.float32: DTYPE_F32,
    torch.int32: DTYPE_I32,
    torch.int64: DTYPE_I64,
    torch.float8_e4m3fn: DTYPE_FP8_E4M3,
    torch.float8_e5m2: DTYPE_FP8_E5M2,
    torch.int8: DTYPE_I8,
}

EXPORTED_SYMBOLS = (
    "b200_abi_version",
    "b200_last_error",
    "b200_choose_num_splits",
    "b200_attn_workspace_bytes",
    "b200_attn_shape_supported",
    "b200_paged_attn_fwd",
    "b200_split_combine",
    "b200_paged_attn_fwd_noalloc",
    "b200_rope_kv_write",
    "b200_kv_cache_write",
    "b200_kv_dequant_pages",
    "b200_device_error",
    "b200_wait_selftest",
)

c_void_p = ctypes.c_void_p
i64 = ctypes.c_int64
i32 = ctypes.c_int32


class AttnParams(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("out", c_void_p),
        ("block_table", c_void_p), ("cu_seqlens_q", c_void_p), ("seqused_k", c_void_p),
        ("q_stride_t", i64), ("q_stride_h", i64),
        ("k_stride_block", i64), ("k_stride_tok", i64), ("k_stride_head", i64),
        ("v_stride_block", i64), ("v_stride_tok", i64), ("v_stride_head", i64),
        ("out_stride_t", i64), ("out_stride_h", i64),
        ("block_table_stride", i64),
        ("block_table_cols", i32), ("block_table_dtype", i32), ("seqlen_dtype", i32), ("dtype", i32),
        ("num_seqs", i32), ("total_q", i32), ("num_q_heads", i32), ("num_kv_heads", i32),
        ("head_dim", i32), ("block_size", i32), ("num_blocks", i32),
        ("max_seqlen_q", i32), ("max_seqlen_k", i32), ("num_splits", i32),
        ("softmax_scale", ctypes.c_float),
        ("workspace", c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class CombineParams(ctypes.Structure):
    _fields_ = [
        ("o_splits", c_void_p), ("m_splits", c_void_p), ("l_splits", c_void_p), ("out", c_void_p),
        ("o_stride_s", i64), ("o_stride_t", i64), ("o_stride_h", i64),
        ("m_stride_s", i64), ("m_stride_t", i64), ("m_stride_h", i64),
        ("l_stride_s", i64), ("l_stride_t", i64), ("l_stride_h", i64),
        ("out_stride_t", i64), ("out_stride_h", i64),
        ("o_dtype", i32), ("out_dtype", i32), ("num_splits", i32), ("total_q", i32),
        ("num_heads", i32), ("head_dim", i32),
    ]


class RopeParams(ctypes.Structure):
    _fields_ = [
        ("query", c_void_p), ("key", c_void_p), ("value", c_void_p), ("positions", c_void_p),
        ("cos_sin_cache", c_void_p), ("key_cache", c_void_p), ("value_cache", c_void_p), ("slot_mapping", c_void_p),
        ("q_stride_t", i64), ("q_stride_h", i64), ("q_stride_d", i64),
        ("k_stride_t", i64), ("k_stride_h", i64), ("k_stride_d", i64),
        ("v_stride_t", i64), ("v_stride_h", i64), ("v_stride_d", i64),
        ("cos_sin_stride_t", i64),
        ("cache_stride_block", i64), ("cache_stride_tok", i64), ("cache_stride_head", i64), ("cache_stride_d", i64),
        ("num_tokens", i32), ("num_q_heads", i32), ("num_kv_heads", i32), ("head_dim", i32),
        ("rotary_dim", i32), ("block_size", i32), ("num_blocks", i32), ("max_position", i32),
        ("is_neox", i32), ("dtype", i32), ("cos_sin_dtype", i32), ("position_dtype", i32), ("slot_dtype", i32),
        ("key_out", c_void_p), ("ko_stride_t", i64), ("ko_stride_h", i64),
        ("cache_dtype", i32), ("k_scale", c_void_p), ("v_scale", c_void_p),
    ]


class KvWriteParams(ctypes.Structure):
    _fields_ = [
        ("key", c_void_p), ("value", c_void_p), ("key_cache", c_void_p), ("value_cache", c_void_p),
        ("slot_mapping", c_void_p), ("k_scale", c_void_p), ("v_scale", c_void_p),
        ("k_scale_cache", c_void_p), ("v_scale_cache", c_void_p),
        ("k_stride_t", i64), ("k_stride_h", i64), ("v_stride_t", i64), ("v_stride_h", i64),
        ("kc_stride_block", i64), ("kc_stride_tok", i64), ("kc_stride_head", i64),
        ("vc_stride_block", i64), ("vc_stride_tok", i64), ("vc_stride_head", i64),
        ("ks_stride_block", i64), ("ks_stride_tok", i64), ("ks_stride_head", i64),
        ("vs_stride_block", i64), ("vs_stride_tok", i64), ("vs_stride_head", i64),
        ("num_tokens", i32), ("num_kv_heads", i32), ("head_dim", i32), ("block_size", i32), ("num_blocks", i32),
        ("dtype", i32), ("cache_dtype", i32), ("quant_mode", i32), ("slot_dtype", i32),
    ]


class KvDequantParams(ctypes.Structure):
    _fields_ = [
        ("key_cache", c_void_p), ("value_cache", c_void_p),
        ("kc_stride_block", i64), ("kc_stride_tok", i64), ("kc_stride_head", i64),
        ("vc_stride_block", i64), ("vc_stride_tok", i64), ("vc_stride_head", i64),
        ("k_scale", c_void_p), ("v_scale", c_void_p), ("k_scale_cache", c_void_p), ("v_scale_cache", c_void_p),
        ("ks_stride_block", i64), ("ks_stride_tok", i64), ("ks_stride_head", i64),
        ("vs_stride_block", i64), ("vs_stride_tok", i64), ("vs_stride_head", i64),
        ("block_table", c_void_p), ("block_table_stride", i64), ("block_table_cols", i32), ("block_table_dtype", i32),
        ("seqused_k", c_void_p), ("seqlen_dtype", i32),
        ("out_cache", c_void_p), ("out_block_table", c_void_p),
        ("num_seqs", i32), ("max_pages", i32), ("block_size", i32), ("num_kv_heads", i32), ("head_dim", i32),
        ("num_blocks", i32), ("cache_dtype", i32), ("quant_mode", i32), ("out_dtype", i32),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once; raise ``RuntimeError`` if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("MINICPM_B200_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"sm_100a library not found at {path}; build it with "
                "`python minicpm-attention-optimization-iluvatar_b200/build.py`"
            )
        lib = ctypes.CDLL(str(path))
        lib.b200_abi_version.restype = ctypes.c_int
        lib.b200_last_error.restype = ctypes.c_char_p
        lib.b200_choose_num_splits.restype = i32
        lib.b200_choose_num_splits.argtypes = [i32] * 5
        lib.b200_attn_workspace_bytes.restype = ctypes.c_size_t
        lib.b200_attn_workspace_bytes.argtypes = [i32] * 8
        lib.b200_attn_shape_supported.restype = i32
        lib.b200_attn_shape_supported.argtypes = [i32] * 4
        lib.b200_paged_attn_fwd.restype = ctypes.c_int
        lib.b200_paged_attn_fwd.argtypes = [ctypes.POINTER(AttnParams), c_void_p]
        lib.b200_split_combine.restype = ctypes.c_int
        lib.b200_split_combine.argtypes = [ctypes.POINTER(CombineParams), c_void_p]
        lib.b200_rope_kv_write.restype = ctypes.c_int
        lib.b200_rope_kv_write.argtypes = [ctypes.POINTER(RopeParams), c_void_p]
        lib.b200_paged_attn_fwd_noalloc.restype = ctypes.c_int
        lib.b200_paged_attn_fwd_noalloc.argtypes = [ctypes.POINTER(AttnParams), c_void_p]
        lib.b200_kv_cache_write.restype = ctypes.c_int
        lib.b200_kv_cache_write.argtypes = [ctypes.POINTER(KvWriteParams), c_void_p]
        lib.b200_kv_dequant_pages.restype = ctypes.c_int
        lib.b200_kv_dequant_pages.argtypes = [ctypes.POINTER(KvDequantParams), c_void_p]
        lib.b200_device_error.restype = ctypes.c_int
        lib.b200_device_error.argtypes = [c_void_p, ctypes.POINTER(ctypes.c_uint32)]
        lib.b200_wait_selftest.restype = ctypes.c_int
        lib.b200_wait_selftest.argtypes = [c_void_p]
        if lib.b200_abi_version() != ABI_VERSION:
            raise RuntimeError("libminicpm_b200.so ABI version mismatch; rebuild it")
        _lib = lib
    return _lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _TORCH_DTYPES[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {dtype}") from exc


def check(status: int, what: str) -> None:
    """Map a C status to the reference's exception types."""
    if status == B200_OK:
        return
    msg = load().b200_last_error().decode(errors="replace")
    if status == B200_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(f"{what}: {msg}")


def current_stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error(device: torch.device | None = None) -> int:
    """Synchronise the current stream and return/clear the library's device error word."""
    lib = load()
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    code = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        check(lib.b200_device_error(current_stream(dev), ctypes.byref(code)), "b200_device_error")
    return int(code.value)


# Workspace buffers cached per (device, stream): calls on one stream are
# ordered, so they can share one buffer; calls on different streams cannot.
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), current_stream(device))
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        if buf is not None:
            size = max(size, int(buf.numel() * 1.25))
        buf = torch.empty(size, dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf
