"""The vLLM-ABI attention dispatcher, in front of the sm_100a kernel.

Mirrors ``iluvatar_attention`` of the reference (``kernels/attention.py:29-167``):
same signature, same feature guards, same routing, same exceptions.

* ``k``/``v`` given as the 5-D ``[blocks, 2, block, kv_heads, D]`` cache are
  unbound to ``k[:, 0]`` and ``v[:, 1]`` (``kernels/attention.py:93-96``).
* The optimized path is taken when ``ILUVATAR_USE_OPTIMIZED=1`` and
  ``ILUVATAR_SPLIT_KV=1`` and none of the unsupported features is requested
  (``max_seqlen_q <= 1``, softcap, ALiBi, a sliding window, ``q_descale``,
  sinks, ``use_td``); failures on that path propagate,
  there is no silent fallback (``kernels/attention.py:151-152``).
* A quantised cache (``kv_quant_mode`` 1: fp8 per-tensor with
  ``k_descale`` / ``v_descale``; 2 / 3: int8 / fp8 per-token-head with the
  scale caches) takes the optimized path too: its referenced pages are
  dequantised (``b200_kv_dequant_pages``) and attended by the same kernel.
  The reference routes every quantised cache to vLLM.
* A head shape or element type the sm_100a kernel does not run (fp32,
  head_dim other than 64 / 128 / 256, more than 128 query heads per KV head;
  ``kernel_supports``)
  is routed like an unsupported feature: the reference's Triton kernel took
  these shapes, so they must not turn into an error here.
* Otherwise the call goes to vLLM's ``unified_attention``, as in the
  reference, and ``RuntimeError`` is raised when vLLM is not importable
  (``kernels/attention.py:112-117``).  That route is vLLM's own kernel and is
  not part of this package.

Differences: the two enable flags are read at every call rather than once at
import (the reference's service twin reads them per call too), so a process
can switch paths without re-importing.  ``ILUVATAR_NUM_SPLITS`` unset means
an automatically chosen split count instead of 4.  ``ILUVATAR_SPLIT_KV_DECODE=1``
(new, off by default, so the reference's routing is kept unless asked for)
sends pure-decode calls (``max_seqlen_q == 1``) to the sm_100a decode kernel
instead of vLLM; the reference left decode on vLLM and its own decode
experiment (``experiments/patches/2026-10-09-native-decode-unvalidated.patch``)
was never validated.
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from .split_kv_paged import kernel_supports
from .unified_attention_optimized import unified_attention_optimized


def _flag(name: str) -> bool:
    return os.environ.get(name, "0") == "1"


def use_optimized() -> bool:
    return _flag("ILUVATAR_USE_OPTIMIZED")


def split_kv_enabled() -> bool:
    return _flag("ILUVATAR_SPLIT_KV")


def decode_enabled() -> bool:
    return _flag("ILUVATAR_SPLIT_KV_DECODE")


def _vllm_unified_attention():
    try:
        from vllm.v1.attention.ops.triton_unified_attention import unified_attention
    except Exception:  # vLLM missing or broken: the reference treats both as unavailable
        return None
    return unified_attention


def _quantised_cache_supported(kv_quant_mode, k_descale, v_descale, k_scale_cache, v_scale_cache) -> bool:
    """A quantised cache the sm_100a path dequantises: fp8 per-tensor with its
    descales, or int8 / fp8 per-token-head with the scale caches (vLLM's
    KVQuantMode 1 / 2 / 3)."""
    mode = int(kv_quant_mode)
    if mode == 0:
        return True
    if mode == 1:
        return k_descale is not None and v_descale is not None
    if mode in (2, 3):
        return k_scale_cache is not None and v_scale_cache is not None
    return False


def iluvatar_attention(
    # Standard vLLM attention API
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    out: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    max_seqlen_q: int,
    seqused_k: torch.Tensor,
    max_seqlen_k: int,
    softmax_scale: float,
    causal: bool = True,
    window_size: tuple = (-1, -1),
    block_table: Optional[torch.Tensor] = None,
    softcap: float = 0.0,
    q_descale: Optional[torch.Tensor] = None,
    k_descale: Optional[torch.Tensor] = None,
    v_descale: Optional[torch.Tensor] = None,
    # Split-KV parameters
    seq_threshold_3D: Optional[int] = None,
    num_par_softmax_segments: Optional[int] = None,
    softmax_segm_output: Optional[torch.Tensor] = None,
    softmax_segm_max: Optional[torch.Tensor] = None,
    softmax_segm_expsum: Optional[torch.Tensor] = None,
    # Additional parameters
    alibi_slopes: Optional[torch.Tensor] = None,
    output_scale: Optional[torch.Tensor] = None,
    qq_bias: Optional[torch.Tensor] = None,
    sinks: Optional[torch.Tensor] = None,
    mm_prefix_range: Optional[tuple] = None,
    use_alibi_sqrt: bool = False,
    kv_quant_mode: int = 0,
    k_scale_cache: Optional[torch.Tensor] = None,
    v_scale_cache: Optional[torch.Tensor] = None,
    chunk_lookback: int = -1,
    use_td: bool = False,
    # Optimization overrides (from harness)
    block_m_override: Optional[int] = None,
    launch_num_warps_override: Optional[int] = None,
    launch_num_stages_override: Optional[int] = None,
    # RoPE parameters
    cos_cache: Optional[torch.Tensor] = None,
    sin_cache: Optional[torch.Tensor] = None,
    rotary_dim: Optional[int] = None,
) -> torch.Tensor:
    """Route one attention call; returns ``out`` (written in place)."""
    original_k, original_v = k, v
    if k.ndim == 5 and v.ndim == 5:
        k, v = k[:, 0], v[:, 1]

    use_baseline = (
        not use_optimized()
        or not split_kv_enabled()
        or max_seqlen_q < 1
        or (max_seqlen_q == 1 and not decode_enabled())
        or softcap != 0.0
        or not _quantised_cache_supported(kv_quant_mode, k_descale, v_descale, k_scale_cache, v_scale_cache)
        or alibi_slopes is not None
        or window_size != (-1, -1)
        or q_descale is not None
        or sinks is not None
        or use_td
        or not kernel_supports(q, k, kv_quant_mode)
    )

    if use_baseline:
        unified_attention = _vllm_unified_attention()
        if unified_attention is None:
            raise RuntimeError(
                "Optimized path disabled and vLLM baseline unavailable. "
                "Enable optimizations with ILUVATAR_USE_OPTIMIZED=1"
            )
        return unified_attention(
            q=q, k=original_k, v=original_v, out=out,
            cu_seqlens_q=cu_seqlens_q,
            max_seqlen_q=max_seqlen_q,
            seqused_k=seqused_k,
            max_seqlen_k=max_seqlen_k,
            softmax_scale=softmax_scale,
            causal=causal,
            window_size=window_size,
            block_table=block_table,
            softcap=softcap,
            q_descale=q_descale,
            k_descale=k_descale,
            v_descale=v_descale,
            seq_threshold_3D=seq_threshold_3D,
            num_par_softmax_segments=num_par_softmax_segments,
            softmax_segm_output=softmax_segm_output,
            softmax_segm_max=softmax_segm_max,
            softmax_segm_expsum=softmax_segm_expsum,
            alibi_slopes=alibi_slopes,
            output_scale=output_scale,
            qq_bias=qq_bias,
            sinks=sinks,
            mm_prefix_range=mm_prefix_range,
            use_alibi_sqrt=use_alibi_sqrt,
            kv_quant_mode=kv_quant_mode,
            k_scale_cache=k_scale_cache,
            v_scale_cache=v_scale_cache,
            chunk_lookback=chunk_lookback,
            use_td=use_td,
        )

    return unified_attention_optimized(
        q=q, k=k, v=v, out=out,
        block_table=block_table,
        seqused_k=seqused_k,
        cu_seqlens_q=cu_seqlens_q,
        max_seqlen_q=max_seqlen_q,
        max_seqlen_k=max_seqlen_k,
        softmax_scale=softmax_scale,
        causal=causal,
        block_m_override=block_m_override or int(os.environ.get("ILUVATAR_BLOCK_M", "64")),
        block_n_override=int(os.environ.get("ILUVATAR_BLOCK_N", "64")),
        launch_num_warps_override=launch_num_warps_override or int(os.environ.get("ILUVATAR_NUM_WARPS", "4")),
        launch_num_stages_override=launch_num_stages_override or int(os.environ.get("ILUVATAR_NUM_STAGES", "2")),
        num_splits_override=int(os.environ.get("ILUVATAR_NUM_SPLITS", "0") or 0),
        kv_quant_mode=kv_quant_mode,
        k_descale=k_descale,
        v_descale=v_descale,
        k_scale_cache=k_scale_cache,
        v_scale_cache=v_scale_cache,
    )


__all__ = ["iluvatar_attention"]
