"""Compatibility entry point in front of the sm_100a Split-KV attention.

Mirrors ``unified_attention_optimized`` of the reference
(``kernels/triton_unified_attention_optimized.py:13-52``): rejects
non-causal calls with ``ValueError``, resolves the split count from the
override, then ``ILUVATAR_NUM_SPLITS``, then
``VLLM_ILUVATAR_ATTN_SPLIT_KV_SEGMENTS``, and swallows extra keyword
arguments.  Differences: when none of the three is set the split count
is chosen automatically (``0``) instead of the reference's fixed 4; and a
quantised cache (``kv_quant_mode`` 1: fp8 per-tensor with ``k_descale`` /
``v_descale``; 2 / 3: int8 / fp8 per-token-head with ``k_scale_cache`` /
``v_scale_cache``), which the reference leaves to vLLM, is dequantised page by
page (``b200_kv_dequant_pages``) and attended by the same kernel.
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from .kv_cache import dequantize_kv_pages
from .split_kv_paged import paged_split_kv_attention


def resolve_num_splits(override: Optional[int]) -> int:
    if override:
        return int(override)
    env = int(os.environ.get("ILUVATAR_NUM_SPLITS", "0") or 0)
    if env:
        return env
    return int(os.environ.get("VLLM_ILUVATAR_ATTN_SPLIT_KV_SEGMENTS", "0") or 0)


def unified_attention_optimized(
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
    causal: bool = True,
    num_splits_override: Optional[int] = None,
    block_m_override: Optional[int] = None,
    block_n_override: Optional[int] = None,
    launch_num_warps_override: Optional[int] = None,
    launch_num_stages_override: Optional[int] = None,
    kv_quant_mode: int = 0,
    k_descale: Optional[torch.Tensor] = None,
    v_descale: Optional[torch.Tensor] = None,
    k_scale_cache: Optional[torch.Tensor] = None,
    v_scale_cache: Optional[torch.Tensor] = None,
    **kwargs,
) -> torch.Tensor:
    if causal is not True:
        raise ValueError("Split-KV currently supports causal attention only")
    if kv_quant_mode:
        # A quantised cache: the referenced pages dequantised into a dense
        # cache in the query dtype, then the same kernel.
        dense, block_table = dequantize_kv_pages(
            k, v, block_table, seqused_k, max_seqlen_k, kv_quant_mode, q.dtype, q.shape[2],
            k_descale=k_descale, v_descale=v_descale, k_scale_cache=k_scale_cache, v_scale_cache=v_scale_cache)
        k, v = dense[:, 0], dense[:, 1]
    return paged_split_kv_attention(
        q=q,
        k=k,
        v=v,
        out=out,
        block_table=block_table,
        seqused_k=seqused_k,
        cu_seqlens_q=cu_seqlens_q,
        max_seqlen_q=max_seqlen_q,
        max_seqlen_k=max_seqlen_k,
        softmax_scale=softmax_scale,
        num_splits=resolve_num_splits(num_splits_override),
        block_m=block_m_override or 64,
        block_n=block_n_override or 64,
        num_warps=launch_num_warps_override or 4,
        num_stages=launch_num_stages_override or 2,
    )


__all__ = ["unified_attention_optimized", "resolve_num_splits"]
