"""Paged KV-cache updates of the serving path on sm_100a.

The reference's service shim updates the cache in two ways
(``integration/vllm-plugin-FL-split-kv.patch``):

* ``IluvatarAttentionImpl.do_kv_cache_update`` (:815-858) calls vLLM's
  ``triton_reshape_and_cache_flash`` (plain and fp8 per-tensor caches) or
  ``triton_reshape_and_cache_flash_per_token_head_quant`` (int8 / fp8 caches
  with one dynamic scale per token and head).  :func:`reshape_and_cache_flash`
  and :func:`reshape_and_cache_flash_per_token_head_quant` take the same
  arguments (``vllm/v1/attention/ops/triton_reshape_and_cache_flash.py``,
  vLLM 0.22) and run ``b200_kv_cache_write``.
* ``IluvatarAttentionImpl.do_rope_and_kv_cache_update`` (:865-899) calls the
  fused rope-and-cache operator with ``q_out = query`` and ``k_out = key``:
  query and key are rotated in place and the caches receive the rotated key
  (quantised with ``k_scale`` / ``v_scale`` when the cache is fp8).
  :func:`rope_and_cache` takes the same arguments as vLLM's
  ``rocm_aiter_ops.triton_rope_and_cache`` and runs ``b200_rope_kv_write`` with
  ``key_out``.

Only the "flash" (NHD) cache layout ``[num_blocks, block_size, kv_heads,
head_dim]`` is handled; it is the only layout the service passes.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

# Per-token-head quantisation: cache dtype -> kv-quant mode (the QUANT_MAX /
# QUANT_MIN pairs are fixed by the mode: int8 127 / -128, fp8 e4m3 448 / -448).
_PER_TOKEN_HEAD_MODES = {
    torch.int8: _lib.KVQ_INT8_PER_TOKEN_HEAD,
    torch.float8_e4m3fn: _lib.KVQ_FP8_PER_TOKEN_HEAD,
}

# vLLM's fp8 dtype on CUDA (``current_platform.fp8_dtype()``): the per-tensor
# fp8 cache is written in e4m3 whatever dtype the cache tensor was allocated with.
FP8_DTYPE = torch.float8_e4m3fn


def is_quantized_kv_cache(kv_cache_dtype: str) -> bool:
    """vLLM's rule (``vllm/v1/kv_cache_interface.py``): fp8*, *per_token_head, nvfp4."""
    return kv_cache_dtype.startswith("fp8") or kv_cache_dtype.endswith("per_token_head") or kv_cache_dtype == "nvfp4"


def _check_common(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    if key.ndim != 3 or value.ndim != 3:
        raise ValueError("key/value must have shape [tokens, kv_heads, head_dim]")
    if key_cache.ndim != 4 or value_cache.ndim != 4:
        raise ValueError("only the flash (NHD) cache layout [num_blocks, block_size, kv_heads, head_dim] is supported")
    if value.shape != key.shape:
        raise ValueError("key/value shapes must match")
    if key_cache.shape != value_cache.shape:
        raise ValueError("key/value cache shapes must match")
    if key_cache.shape[2] != key.shape[1] or key_cache.shape[3] < key.shape[2]:
        raise ValueError("cache shape does not match key/value")
    if slot_mapping.ndim != 1 or slot_mapping.shape[0] != key.shape[0]:
        raise ValueError("slot_mapping must have one entry per token")
    if slot_mapping.dtype not in (torch.int32, torch.int64):
        raise ValueError("slot_mapping must contain int32 or int64 indices")
    dev = key.device
    for t in (value, key_cache, value_cache, slot_mapping):
        if t.device != dev:
            raise ValueError("all tensors must be on the key's device")
    if dev.type != "cuda":
        raise RuntimeError("KV-cache writes run on CUDA tensors only (no CPU path)")
    if key.dtype not in (torch.float16, torch.bfloat16, torch.float32) or value.dtype != key.dtype:
        raise ValueError("key/value must share a float16, bfloat16 or float32 dtype")
    if key.shape[2] not in (64, 128, 256):
        raise ValueError("head_dim must be 64, 128 or 256")
    for t in (key, value, key_cache, value_cache):
        if t.stride(-1) != 1:
            raise ValueError("head_dim must be contiguous")


def _launch(params: _lib.KvWriteParams, device: torch.device, what: str) -> None:
    lib = _lib.load()
    with torch.cuda.device(device):
        _lib.check(lib.b200_kv_cache_write(ctypes.byref(params), _lib.current_stream(device)), what)


def _params(key, value, key_cache, value_cache, slot_mapping, cache_dtype_code, mode, **extra) -> _lib.KvWriteParams:
    # A non-contiguous slot_mapping is compacted; the copy is freed after the
    # launch is queued, which the caching allocator orders behind it on this stream.
    slot_mapping = slot_mapping.contiguous()
    return _lib.KvWriteParams(
        key=key.data_ptr(), value=value.data_ptr(), key_cache=key_cache.data_ptr(), value_cache=value_cache.data_ptr(),
        slot_mapping=slot_mapping.data_ptr(),
        k_stride_t=key.stride(0), k_stride_h=key.stride(1), v_stride_t=value.stride(0), v_stride_h=value.stride(1),
        kc_stride_block=key_cache.stride(0), kc_stride_tok=key_cache.stride(1), kc_stride_head=key_cache.stride(2),
        vc_stride_block=value_cache.stride(0), vc_stride_tok=value_cache.stride(1), vc_stride_head=value_cache.stride(2),
        num_tokens=key.shape[0], num_kv_heads=key.shape[1], head_dim=key.shape[2],
        block_size=key_cache.shape[1], num_blocks=key_cache.shape[0],
        dtype=_lib.dtype_code(key.dtype), cache_dtype=cache_dtype_code, quant_mode=mode,
        slot_dtype=_lib.dtype_code(slot_mapping.dtype), **extra,
    )


def _scalar_scale(scale: torch.Tensor, device: torch.device, name: str) -> torch.Tensor:
    if not isinstance(scale, torch.Tensor) or scale.numel() < 1:
        raise ValueError(f"{name} must be a float32 tensor with one element")
    if scale.device != device:
        raise ValueError(f"{name} must be on the key's device")
    if scale.dtype != torch.float32:
        raise ValueError(f"{name} must be float32")
    return scale.reshape(-1)[:1].contiguous()


def reshape_and_cache_flash(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    kv_cache_dtype: str,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
) -> None:
    """Write ``key``/``value`` ``[T, KH, D]`` into the paged caches at ``slot_mapping``.

    ``kv_cache_dtype`` "auto": the caches have the key dtype and receive its
    bits.  fp8 kinds ("fp8", "fp8_e4m3", "fp8_e5m2"): the caches (fp8 or uint8
    storage) receive ``fp8_e4m3(x / scale)``, round-to-nearest-even and
    saturating.  Tokens with a negative slot are skipped.
    """
    if not (kv_cache_dtype == "auto" or is_quantized_kv_cache(kv_cache_dtype)):
        raise AssertionError(f"unsupported kv_cache_dtype (str), got {kv_cache_dtype}.")
    if kv_cache_dtype.endswith("per_token_head") or kv_cache_dtype == "nvfp4":
        raise ValueError(f"kv_cache_dtype {kv_cache_dtype} is not written by reshape_and_cache_flash")
    _check_common(key, value, key_cache, value_cache, slot_mapping)
    if key.shape[0] == 0:
        return None
    if kv_cache_dtype == "auto":
        if key_cache.dtype != key.dtype or value_cache.dtype != key.dtype:
            raise ValueError("an unquantised cache must have the key dtype")
        if key_cache.shape[3] != key.shape[2]:
            raise ValueError("cache head_dim must equal the key head_dim")
        p = _params(key, value, key_cache, value_cache, slot_mapping, _lib.dtype_code(key.dtype), _lib.KVQ_NONE)
        _launch(p, key.device, "reshape_and_cache_flash")
        return None
    if key_cache.dtype not in (torch.float8_e4m3fn, torch.float8_e5m2, torch.uint8):
        raise AssertionError(
            f"unsupported dtype of KV cache tensor, got {key_cache.dtype}. "
            "Supported kv cache dtypes: fp8e4m3fn, fp8e5m2, uint8."
        )
    if value_cache.dtype != key_cache.dtype:
        raise ValueError("key/value caches must share a dtype")
    ks = _scalar_scale(k_scale, key.device, "k_scale")
    vs = _scalar_scale(v_scale, key.device, "v_scale")
    p = _params(
        key, value, key_cache, value_cache, slot_mapping, _lib.DTYPE_FP8_E4M3, _lib.KVQ_FP8_PER_TENSOR,
        k_scale=ks.data_ptr(), v_scale=vs.data_ptr(),
    )
    _launch(p, key.device, "reshape_and_cache_flash")
    return None


def reshape_and_cache_flash_per_token_head_quant(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    k_scale_cache: torch.Tensor,
    v_scale_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Quantise each (token, head) of ``key``/``value`` with its own scale.

    ``s = max(max|x| / QMAX, 1e-6)``, ``q = clamp(x * (1 / s), QMIN, QMAX)``;
    int8 caches truncate toward zero (QMAX 127, QMIN -128), fp8 e4m3 caches
    round to nearest even (+-448).  ``s`` goes to ``k_scale_cache`` /
    ``v_scale_cache`` ``[num_blocks, block_size, kv_heads]`` (float32, any
    strides -- typically views into the inline padding of the cache rows).
    """
    mode = _PER_TOKEN_HEAD_MODES.get(key_cache.dtype)
    if mode is None:
        raise ValueError(
            f"Per-token-head quantization not supported for cache dtype {key_cache.dtype}.  "
            f"Supported: {list(_PER_TOKEN_HEAD_MODES)}"
        )
    _check_common(key, value, key_cache, value_cache, slot_mapping)
    if value_cache.dtype != key_cache.dtype:
        raise ValueError("key/value caches must share a dtype")
    for name, sc in (("k_scale_cache", k_scale_cache), ("v_scale_cache", v_scale_cache)):
        if sc.dtype != torch.float32 or sc.ndim != 3 or tuple(sc.shape) != tuple(key_cache.shape[:3]):
            raise ValueError(f"{name} must be float32 [num_blocks, block_size, kv_heads]")
        if sc.device != key.device:
            raise ValueError(f"{name} must be on the key's device")
    if key.shape[0] == 0:
        return None
    p = _params(
        key, value, key_cache, value_cache, slot_mapping, _lib.dtype_code(key_cache.dtype), mode,
        k_scale_cache=k_scale_cache.data_ptr(), v_scale_cache=v_scale_cache.data_ptr(),
        ks_stride_block=k_scale_cache.stride(0), ks_stride_tok=k_scale_cache.stride(1),
        ks_stride_head=k_scale_cache.stride(2),
        vs_stride_block=v_scale_cache.stride(0), vs_stride_tok=v_scale_cache.stride(1),
        vs_stride_head=v_scale_cache.stride(2),
    )
    _launch(p, key.device, "reshape_and_cache_flash_per_token_head_quant")
    return None


def rope_and_cache(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    is_neox: bool,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    flash_layout: bool,
    apply_scale: bool,
) -> None:
    """The service's fused RoPE + cache update (``q_out = query``, ``k_out = key``).

    ``query`` and ``key`` are rotated in place for every token; tokens with a
    non-negative slot write the rotated key and the value into the caches, as
    ``fp8_e4m3(x / scale)`` when ``apply_scale`` (fp8 caches), else unchanged.
    """
    if not flash_layout:
        raise NotImplementedError("only the flash (NHD) KV-cache layout is supported")
    if query.ndim != 3 or key.ndim != 3 or value.ndim != 3:
        raise ValueError("query/key/value must have shape [tokens, heads, head_dim]")
    if query.dtype not in (torch.bfloat16, torch.float16) or key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError("query/key/value must share a bfloat16 or float16 dtype")
    _check_common(key, value, key_cache, value_cache, slot_mapping)
    if query.device != key.device or positions.device != key.device or cos_sin_cache.device != key.device:
        raise ValueError("all tensors must be on the key's device")
    if key_cache.stride() != value_cache.stride():
        raise ValueError("key/value cache strides must match")
    if positions.dtype not in (torch.int32, torch.int64) or positions.numel() != query.shape[0]:
        raise ValueError("positions must hold one integer index per token")
    if cos_sin_cache.ndim != 2 or cos_sin_cache.shape[1] % 2 or cos_sin_cache.shape[1] > query.shape[2]:
        raise ValueError("cos_sin_cache must be [max_position, rotary_dim]")
    if cos_sin_cache.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError("cos_sin_cache must be f16, bf16 or f32")
    if key.shape[0] != query.shape[0] or query.shape[2] != key.shape[2] or query.shape[1] < key.shape[1]:
        raise ValueError("query/key shapes do not match")
    if key_cache.shape[3] != key.shape[2]:
        raise ValueError("cache head_dim must equal the key head_dim")
    extra = {}
    if apply_scale:
        if key_cache.dtype not in (torch.float8_e4m3fn, torch.float8_e5m2, torch.uint8) or value_cache.dtype != key_cache.dtype:
            raise ValueError("apply_scale requires fp8 (or uint8-stored fp8) caches")
        cache_code = _lib.DTYPE_FP8_E4M3
        extra = dict(k_scale=_scalar_scale(k_scale, key.device, "k_scale").data_ptr(),
                     v_scale=_scalar_scale(v_scale, key.device, "v_scale").data_ptr())
    else:
        if key_cache.dtype != key.dtype or value_cache.dtype != key.dtype:
            raise ValueError("without apply_scale the caches must have the key dtype")
        cache_code = _lib.dtype_code(key.dtype)
    if query.shape[0] == 0:
        return None
    positions = positions.reshape(-1).contiguous()
    slot_mapping = slot_mapping.contiguous()
    if cos_sin_cache.stride(1) != 1:
        cos_sin_cache = cos_sin_cache.contiguous()
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
        num_tokens=query.shape[0], num_q_heads=query.shape[1], num_kv_heads=key.shape[1], head_dim=query.shape[2],
        rotary_dim=cos_sin_cache.shape[1], block_size=key_cache.shape[1], num_blocks=key_cache.shape[0],
        max_position=cos_sin_cache.shape[0], is_neox=int(bool(is_neox)),
        dtype=_lib.dtype_code(query.dtype), cos_sin_dtype=_lib.dtype_code(cos_sin_cache.dtype),
        position_dtype=_lib.dtype_code(positions.dtype), slot_dtype=_lib.dtype_code(slot_mapping.dtype),
        key_out=key.data_ptr(), ko_stride_t=key.stride(0), ko_stride_h=key.stride(1),
        cache_dtype=cache_code, **extra,
    )
    lib = _lib.load()
    with torch.cuda.device(query.device):
        _lib.check(lib.b200_rope_kv_write(ctypes.byref(p), _lib.current_stream(query.device)), "rope_and_cache")
    return None


__all__ = [
    "dequantize_kv_pages",
    "FP8_DTYPE",
    "is_quantized_kv_cache",
    "reshape_and_cache_flash",
    "reshape_and_cache_flash_per_token_head_quant",
    "rope_and_cache",
]


# ---------------------------------------------------------------------------
# Attention over quantised caches: the referenced pages, dequantised.
# ---------------------------------------------------------------------------

_DEQUANT_ELEM = {torch.float8_e4m3fn: _lib.DTYPE_FP8_E4M3, torch.float8_e5m2: _lib.DTYPE_FP8_E5M2,
                 torch.int8: _lib.DTYPE_I8, torch.uint8: _lib.DTYPE_FP8_E4M3}

# Dense dequantised caches cached per (device, stream): calls on one stream are
# ordered, so they can share one buffer.
_dense: dict[tuple[int, int], torch.Tensor] = {}


def dequantize_kv_pages(key_cache: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
                        seqused_k: torch.Tensor, max_seqlen_k: int, kv_quant_mode: int, out_dtype: torch.dtype,
                        head_dim: int, k_descale: torch.Tensor | None = None, v_descale: torch.Tensor | None = None,
                        k_scale_cache: torch.Tensor | None = None, v_scale_cache: torch.Tensor | None = None
                        ) -> tuple[torch.Tensor, torch.Tensor]:
    """The pages ``block_table`` references, dequantised into a dense cache.

    For the attention calls the reference's service makes on quantised caches
    (``kv_quant_mode`` 1: fp8 per-tensor with ``k_descale`` / ``v_descale``,
    whose first element is the scale, as vLLM's ``unified_attention`` reads it;
    2 / 3: int8 / fp8 per-token-head with ``k_scale_cache`` / ``v_scale_cache``
    ``[num_blocks, block_size, kv_heads]`` float views; the cache rows may be
    longer than ``head_dim``, as the service's rows with the scale inline
    are).  Returns ``(cache,
    table)``: ``cache [num_seqs * max_pages, 2, block_size, kv_heads, head_dim]``
    in ``out_dtype`` and ``table [num_seqs, max_pages]`` int32, max_pages =
    ceil(max_seqlen_k / block_size), ready for :func:`paged_split_kv_attention`
    on ``cache[:, 0]`` / ``cache[:, 1]``.  The cache buffer is reused by the next
    call on the same stream.
    """
    if key_cache.ndim != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("expected key/value caches [num_blocks, block_size, kv_heads, >= head_dim]")
    if key_cache.device.type != "cuda":
        raise RuntimeError("dequantize_kv_pages runs on CUDA tensors only (no CPU path)")
    elem = _DEQUANT_ELEM.get(key_cache.dtype)
    if elem is None:
        raise ValueError(f"no dequantisation for a {key_cache.dtype} cache")
    if kv_quant_mode == _lib.KVQ_INT8_PER_TOKEN_HEAD and key_cache.dtype in (torch.int8, torch.uint8):
        elem = _lib.DTYPE_I8
    if kv_quant_mode == _lib.KVQ_FP8_PER_TENSOR:
        if k_descale is None or v_descale is None:
            raise ValueError("fp8 per-tensor caches need k_descale and v_descale")
        k_scale = k_descale.to(device=key_cache.device, dtype=torch.float32).reshape(-1)[:1].contiguous()
        v_scale = v_descale.to(device=key_cache.device, dtype=torch.float32).reshape(-1)[:1].contiguous()
        ksc = vsc = None
    else:
        if k_scale_cache is None or v_scale_cache is None:
            raise ValueError("per-token-head caches need k_scale_cache and v_scale_cache")
        ksc, vsc = k_scale_cache, v_scale_cache
        k_scale = v_scale = None
    num_blocks, block_size, kv_heads, row = key_cache.shape
    if head_dim > row or head_dim % 4 or key_cache.stride(3) != 1:
        raise ValueError("cache rows must hold head_dim contiguous elements")
    num_seqs = int(seqused_k.numel())
    max_pages = max(1, -(-int(max_seqlen_k) // block_size))
    dev = key_cache.device
    n = num_seqs * max_pages * 2 * block_size * kv_heads * head_dim
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), _lib.current_stream(dev))
    buf = _dense.get((key, out_dtype))
    if buf is None or buf.numel() < n:
        buf = torch.empty(max(n, 1), dtype=out_dtype, device=dev)
        _dense[(key, out_dtype)] = buf
    cache = buf[:n].view(num_seqs * max_pages, 2, block_size, kv_heads, head_dim)
    table = torch.empty(num_seqs, max_pages, dtype=torch.int32, device=dev)
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    seqused_k = seqused_k.contiguous()
    p = _lib.KvDequantParams(
        key_cache=key_cache.data_ptr(), value_cache=value_cache.data_ptr(),
        kc_stride_block=key_cache.stride(0), kc_stride_tok=key_cache.stride(1), kc_stride_head=key_cache.stride(2),
        vc_stride_block=value_cache.stride(0), vc_stride_tok=value_cache.stride(1),
        vc_stride_head=value_cache.stride(2),
        k_scale=k_scale.data_ptr() if k_scale is not None else None,
        v_scale=v_scale.data_ptr() if v_scale is not None else None,
        k_scale_cache=ksc.data_ptr() if ksc is not None else None,
        v_scale_cache=vsc.data_ptr() if vsc is not None else None,
        ks_stride_block=ksc.stride(0) if ksc is not None else 0, ks_stride_tok=ksc.stride(1) if ksc is not None else 0,
        ks_stride_head=ksc.stride(2) if ksc is not None else 0,
        vs_stride_block=vsc.stride(0) if vsc is not None else 0, vs_stride_tok=vsc.stride(1) if vsc is not None else 0,
        vs_stride_head=vsc.stride(2) if vsc is not None else 0,
        block_table=block_table.data_ptr(), block_table_stride=block_table.stride(0),
        block_table_cols=block_table.shape[1], block_table_dtype=_lib.dtype_code(block_table.dtype),
        seqused_k=seqused_k.data_ptr(), seqlen_dtype=_lib.dtype_code(seqused_k.dtype),
        out_cache=cache.data_ptr(), out_block_table=table.data_ptr(),
        num_seqs=num_seqs, max_pages=max_pages, block_size=block_size, num_kv_heads=kv_heads, head_dim=head_dim,
        num_blocks=num_blocks, cache_dtype=elem, quant_mode=int(kv_quant_mode), out_dtype=_lib.dtype_code(out_dtype),
    )
    with torch.cuda.device(dev):
        _lib.check(_lib.load().b200_kv_dequant_pages(ctypes.byref(p), _lib.current_stream(dev)), "dequantize_kv_pages")
    return cache, table

