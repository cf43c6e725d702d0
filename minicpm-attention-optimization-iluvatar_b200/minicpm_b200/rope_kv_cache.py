"""Fused RoPE + paged KV-cache write on sm_100a.

Drop-in for ``fused_rope_and_cache`` of the reference
(``kernels/triton_rope_kv_cache.py:205-286``): same signature, validation
messages and in-place effects -- ``query`` rotated in place, rotated ``key``
and unchanged ``value`` written to ``key_cache``/``value_cache`` at
``slot_mapping``, tokens with a negative slot skipped, ``key``/``value``
untouched.  One launch of ``b200_rope_kv_write`` on the current stream.

Stricter than the reference: a position outside ``cos_sin_cache`` or a slot
past the end of the cache is skipped and recorded in the device error word
(``minicpm_b200._lib.device_error()``) instead of being read or written out
of bounds.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def fused_rope_and_cache(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    is_neox: bool,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    rotary_dim: int | None = None,
    num_warps: int = 4,
) -> None:
    """Rotate Q/K and update an NHD paged KV cache in one launch."""
    # Validation mirrors kernels/triton_rope_kv_cache.py:219-260.
    if query.ndim != 3 or key.ndim != 3 or value.ndim != 3:
        raise ValueError("query/key/value must have shape [tokens, heads, head_dim]")
    if key_cache.ndim != 4 or value_cache.ndim != 4:
        raise ValueError("only NHD paged KV cache is supported")
    if query.device != key.device or query.device != value.device:
        raise ValueError("query/key/value must share a device")
    if key_cache.device != query.device or value_cache.device != query.device:
        raise ValueError("cache tensors must share the query device")
    if positions.device != query.device or slot_mapping.device != query.device or cos_sin_cache.device != query.device:
        raise ValueError("positions, slots, and RoPE cache must share the query device")
    if query.dtype != key.dtype or query.dtype != value.dtype:
        raise ValueError("query/key/value must share a dtype")
    if key_cache.shape != value_cache.shape:
        raise ValueError("key/value cache shapes must match")
    if key_cache.stride() != value_cache.stride():
        raise ValueError("key/value cache strides must match")
    if query.dtype not in (torch.bfloat16, torch.float16) or key_cache.dtype != query.dtype or value_cache.dtype != query.dtype:
        raise ValueError("only unquantized BF16/FP16 caches are supported")
    if positions.dtype not in (torch.int32, torch.int64) or slot_mapping.dtype not in (torch.int32, torch.int64):
        raise ValueError("positions and slot_mapping must contain integer indices")
    if positions.numel() != query.shape[0] or slot_mapping.numel() != query.shape[0]:
        raise ValueError("positions and slot_mapping must have one entry per token")
    if cos_sin_cache.ndim != 2 or cos_sin_cache.shape[1] % 2:
        raise ValueError("cos_sin_cache must be [max_position, rotary_dim]")

    tokens, query_heads, head_dim = query.shape
    kv_heads = key.shape[1]
    rotary_dim = rotary_dim or int(cos_sin_cache.shape[1])
    if (
        key.shape[0] != tokens
        or value.shape != key.shape
        or key_cache.shape[2] != kv_heads
        or key_cache.shape[3] != head_dim
        or rotary_dim != cos_sin_cache.shape[1]
        or rotary_dim <= 0
        or rotary_dim > head_dim
        or rotary_dim % 2
        or query_heads < kv_heads
        or head_dim not in (64, 128, 256)
        or key_cache.shape[1] % 16
    ):
        raise ValueError("unsupported RoPE/cache shape")
    if query.device.type != "cuda":
        raise RuntimeError("fused_rope_and_cache runs on CUDA tensors only (no CPU path)")
    if cos_sin_cache.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError("cos_sin_cache must be f16, bf16 or f32")
    if tokens == 0:
        return None
    positions = positions.reshape(-1)
    slot_mapping = slot_mapping.reshape(-1)
    if positions.stride(0) != 1:
        positions = positions.contiguous()
    if slot_mapping.stride(0) != 1:
        slot_mapping = slot_mapping.contiguous()
    if cos_sin_cache.stride(1) != 1:
        cos_sin_cache = cos_sin_cache.contiguous()

    lib = _lib.load()
    p = _lib.RopeParams(
        query=query.data_ptr(), key=key.data_ptr(), value=value.data_ptr(), positions=positions.data_ptr(),
        cos_sin_cache=cos_sin_cache.data_ptr(), key_cache=key_cache.data_ptr(), value_cache=value_cache.data_ptr(),
        slot_mapping=slot_mapping.data_ptr(),
        q_stride_t=query.stride(0), q_stride_h=query.stride(1), q_stride_d=query.stride(2),
        k_stride_t=key.stride(0), k_stride_h=key.stride(1), k_stride_d=key.stride(2),
        v_stride_t=value.stride(0), v_stride_h=value.stride(1), v_stride_d=value.stride(2),
        cos_sin_stride_t=cos_sin_cache.stride(0),
        cache_stride_block=key_cache.stride(0), cache_stride_tok=key_cache.stride(1),
        cache_stride_head=key_cache.stride(2), cache_stride_d=key_cache.stride(3),
        num_tokens=tokens, num_q_heads=query_heads, num_kv_heads=kv_heads, head_dim=head_dim,
        rotary_dim=rotary_dim, block_size=key_cache.shape[1], num_blocks=key_cache.shape[0],
        max_position=cos_sin_cache.shape[0], is_neox=int(bool(is_neox)),
        dtype=_lib.dtype_code(query.dtype), cos_sin_dtype=_lib.dtype_code(cos_sin_cache.dtype),
        position_dtype=_lib.dtype_code(positions.dtype), slot_dtype=_lib.dtype_code(slot_mapping.dtype),
        key_out=None, cache_dtype=_lib.dtype_code(query.dtype),
    )
    with torch.cuda.device(query.device):
        _lib.check(lib.b200_rope_kv_write(ctypes.byref(p), _lib.current_stream(query.device)), "fused_rope_and_cache")
    return None


__all__ = ["fused_rope_and_cache"]
