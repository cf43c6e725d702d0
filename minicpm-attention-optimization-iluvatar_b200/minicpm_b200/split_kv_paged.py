"""Paged Split-KV causal attention on sm_100a.

Drop-in for ``paged_split_kv_attention`` of the reference
(``kernels/triton_split_kv_paged.py:231-361``): same signature, argument
meaning, validation messages and return value.  The work runs in
``libminicpm_b200.so`` (``b200_paged_attn_fwd``): a device-side work list, the
tcgen05 attention kernel and, for ``num_splits > 1``, the split combine, all
on the current CUDA stream and without a host synchronisation.

Differences from the reference, all supersets:

* ``num_splits`` also accepts ``0`` (choose from the SM count and KV length)
  and ``1`` (no split: the kernel writes ``out`` directly, no combine pass);
  other values outside ``{2, 4, 8, 16}`` still raise ``ValueError``.
* ``block_m``, ``block_n``, ``num_warps`` and ``num_stages`` are validated as
  in the reference and otherwise advisory: the kernel's tiles are fixed
  tcgen05 shapes (128 query rows x 128 KV tokens).
* the per-call scratch of the reference (``o_splits``, ``m``, ``l``) lives in a
  workspace cached per device and stream.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_VALID_SPLITS = (0, 1, 2, 4, 8, 16)


def paged_split_kv_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    out: torch.Tensor,
    block_table: torch.Tensor,
    seqused_k: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    max_seqlen_q: int,
    max_seqlen_k: int,
    softmax_scale: float,
    num_splits: int = 4,
    block_m: int = 64,
    block_n: int = 64,
    num_warps: int = 4,
    num_stages: int = 2,
) -> torch.Tensor:
    """Run Split-KV on the exact flattened/paged vLLM attention ABI."""
    # Validation mirrors kernels/triton_split_kv_paged.py:249-281.
    if q.ndim != 3 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("expected q=[T,H,D] and k/v=[blocks,block,kv_heads,D]")
    if q.device != k.device or q.device != v.device or q.device != out.device:
        raise ValueError("q, k, v, and out must be on the same device")
    if out.shape != q.shape or k.shape != v.shape:
        raise ValueError("out must match q and k/v must have identical shapes")
    if num_splits not in _VALID_SPLITS:
        raise ValueError("num_splits must be one of 2, 4, 8, 16")
    if block_table.dtype not in (torch.int32, torch.int64):
        raise ValueError("block_table must contain integer physical block ids")
    if cu_seqlens_q.ndim != 1 or seqused_k.ndim != 1:
        raise ValueError("cu_seqlens_q and seqused_k must be one-dimensional")
    if cu_seqlens_q.numel() != seqused_k.numel() + 1:
        raise ValueError("cu_seqlens_q must contain one entry per request plus one")
    if block_table.shape[0] != seqused_k.numel():
        raise ValueError("block_table and seqused_k must have the same request count")

    total_q, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[2]
    block_size = k.shape[1]
    if (
        head_dim not in (64, 128, 256)
        or num_q_heads % num_kv_heads
        or block_size <= 0
        or block_size % 16
        or block_m <= 0
        or block_m % 16
        or block_n <= 0
        or block_n % 16
    ):
        raise ValueError("unsupported head shape for paged Split-KV")
    if max_seqlen_q <= 0 or max_seqlen_k <= 0:
        return out.zero_()

    if q.device.type != "cuda":
        raise RuntimeError("paged_split_kv_attention runs on CUDA tensors only (no CPU path)")
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype or out.dtype != q.dtype:
        raise RuntimeError("the sm_100a kernel takes bf16 or f16 q/k/v/out of one dtype")
    if q.stride(2) != 1 or k.stride(3) != 1 or v.stride(3) != 1 or out.stride(2) != 1:
        raise RuntimeError("the head dimension of q, k, v and out must be contiguous")
    if cu_seqlens_q.dtype != seqused_k.dtype or cu_seqlens_q.dtype not in (torch.int32, torch.int64):
        raise ValueError("cu_seqlens_q and seqused_k must be int32 or int64 of one dtype")
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    cu_seqlens_q = cu_seqlens_q.contiguous()
    seqused_k = seqused_k.contiguous()

    lib = _lib.load()
    num_seqs = int(seqused_k.numel())
    dtype = _lib.dtype_code(q.dtype)
    nbytes = lib.b200_attn_workspace_bytes(total_q, num_seqs, num_q_heads, num_kv_heads, head_dim, num_splits,
                                           int(max_seqlen_k), dtype)
    ws = _lib.workspace(q.device, nbytes)
    p = _lib.AttnParams(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(),
        block_table=block_table.data_ptr(), cu_seqlens_q=cu_seqlens_q.data_ptr(), seqused_k=seqused_k.data_ptr(),
        q_stride_t=q.stride(0), q_stride_h=q.stride(1),
        k_stride_block=k.stride(0), k_stride_tok=k.stride(1), k_stride_head=k.stride(2),
        v_stride_block=v.stride(0), v_stride_tok=v.stride(1), v_stride_head=v.stride(2),
        out_stride_t=out.stride(0), out_stride_h=out.stride(1),
        block_table_stride=block_table.stride(0), block_table_cols=block_table.shape[1],
        block_table_dtype=_lib.dtype_code(block_table.dtype), seqlen_dtype=_lib.dtype_code(seqused_k.dtype),
        dtype=dtype, num_seqs=num_seqs, total_q=total_q, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads,
        head_dim=head_dim, block_size=block_size, num_blocks=k.shape[0],
        max_seqlen_q=int(max_seqlen_q), max_seqlen_k=int(max_seqlen_k), num_splits=int(num_splits),
        softmax_scale=float(softmax_scale), workspace=ws.data_ptr(), workspace_bytes=ws.numel(),
    )
    with torch.cuda.device(q.device):
        _lib.check(lib.b200_paged_attn_fwd(ctypes.byref(p), _lib.current_stream(q.device)), "paged_split_kv_attention")
    return out


def split_kv_combine(o_splits: torch.Tensor, m_splits: torch.Tensor, l_splits: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """The cross-split reduce of ``_split_kv_reduce`` as its own launch.

    ``o_splits [S, T, H, D]`` (f16/bf16/f32), ``m_splits``/``l_splits [S, T, H]``
    fp32, ``out [T, H, D]`` (f16/bf16/f32), written in place and returned.
    """
    if o_splits.ndim != 4 or m_splits.ndim != 3 or l_splits.ndim != 3 or out.ndim != 3:
        raise ValueError("expected o_splits [S,T,H,D], m/l [S,T,H] and out [T,H,D]")
    if m_splits.shape != o_splits.shape[:3] or l_splits.shape != m_splits.shape or out.shape != o_splits.shape[1:]:
        raise ValueError("o_splits, m, l and out shapes disagree")
    if m_splits.dtype != torch.float32 or l_splits.dtype != torch.float32:
        raise ValueError("m_splits and l_splits must be float32")
    if o_splits.stride(3) != 1 or out.stride(2) != 1:
        raise ValueError("head dimension must be contiguous")
    s, t, h, d = o_splits.shape
    lib = _lib.load()
    p = _lib.CombineParams(
        o_splits=o_splits.data_ptr(), m_splits=m_splits.data_ptr(), l_splits=l_splits.data_ptr(), out=out.data_ptr(),
        o_stride_s=o_splits.stride(0), o_stride_t=o_splits.stride(1), o_stride_h=o_splits.stride(2),
        m_stride_s=m_splits.stride(0), m_stride_t=m_splits.stride(1), m_stride_h=m_splits.stride(2),
        l_stride_s=l_splits.stride(0), l_stride_t=l_splits.stride(1), l_stride_h=l_splits.stride(2),
        out_stride_t=out.stride(0), out_stride_h=out.stride(1),
        o_dtype=_lib.dtype_code(o_splits.dtype), out_dtype=_lib.dtype_code(out.dtype),
        num_splits=s, total_q=t, num_heads=h, head_dim=d,
    )
    with torch.cuda.device(out.device):
        _lib.check(lib.b200_split_combine(ctypes.byref(p), _lib.current_stream(out.device)), "split_kv_combine")
    return out


_QUANT_CACHE_DTYPES = {
    1: (torch.float8_e4m3fn, torch.float8_e5m2, torch.uint8),  # fp8 per-tensor
    2: (torch.int8, torch.uint8),                              # int8 per-token-head
    3: (torch.float8_e4m3fn, torch.uint8),                     # fp8 per-token-head
}


def kernel_supports(q: torch.Tensor, k: torch.Tensor, kv_quant_mode: int = 0) -> bool:
    """Whether the sm_100a kernels run this call's head shape and element types.

    ``q`` is ``[T, Hq, D]``; ``k`` is the 4-D ``[blocks, block, KH, D]`` cache
    or the 5-D ``[blocks, 2, block, KH, D]`` one; a quantised cache
    (``kv_quant_mode`` 1-3) holds 1-byte elements and is dequantised page by
    page first.  The dispatcher and the service route calls for which this is
    false (fp32, head_dim other than 64 / 128 / 256, more than 128 query heads
    per KV head, an unknown quantisation) to their baseline kernel, as they
    route the features the kernels do not implement.
    """
    try:
        code = _lib.dtype_code(q.dtype)
    except ValueError:
        return False
    if q.ndim != 3 or k.ndim not in (4, 5):
        return False
    if kv_quant_mode:
        if k.dtype not in _QUANT_CACHE_DTYPES.get(int(kv_quant_mode), ()):
            return False
    elif k.dtype != q.dtype:
        return False
    return bool(_lib.load().b200_attn_shape_supported(int(q.shape[1]), int(k.shape[-2]), int(q.shape[2]), code))


def choose_num_splits(total_q: int, num_seqs: int, num_q_heads: int, num_kv_heads: int, max_seqlen_k: int) -> int:
    """The split count ``num_splits=0`` resolves to on the current device."""
    return int(_lib.load().b200_choose_num_splits(total_q, num_seqs, num_q_heads, num_kv_heads, max_seqlen_k))


__all__ = ["paged_split_kv_attention", "split_kv_combine", "choose_num_splits", "kernel_supports"]
