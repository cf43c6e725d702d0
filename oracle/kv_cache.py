"""CPU restatement of the service's paged KV-cache updates.

TEST INFRASTRUCTURE ONLY (the checker and the CPU baseline; never shipped).

What is restated (paths inside the reference project, then the third-party
code the reference calls):

* ``integration/vllm-plugin-FL-split-kv.patch:815-858``
  (``IluvatarAttentionImpl.do_kv_cache_update``): which writer runs for which
  ``kv_cache_dtype``, and that the fp8 per-tensor path views the caches as
  float8 e4m3.
* vLLM 0.22 ``vllm/v1/attention/ops/triton_reshape_and_cache_flash.py``
  (not part of the reference project; installed with vLLM):
  ``reshape_and_cache_kernel_flash`` -- a token with ``slot < 0`` writes
  nothing, else ``cache[slot // bs, slot % bs, h, :] = x`` (plain) or
  ``fp8(x / scale)`` (fp8 per-tensor); ``_reshape_cache_per_token_head`` --
  ``s = max(max|x| / QMAX, 1e-6)``, ``q = clamp(x * (1 / s), QMIN, QMAX)``,
  the store's implicit cast (int8: truncation toward zero; fp8: round to
  nearest even), ``s`` to the scale cache.
* ``integration/vllm-plugin-FL-split-kv.patch:865-899``
  (``do_rope_and_kv_cache_update``): rotate query and key in place
  (``q_out = query``, ``k_out = key``) and write the rotated key and the value
  to the caches, fp8 with ``k_scale`` / ``v_scale`` when the cache is fp8.
  The fused operator it calls (AMD aiter's ``fused_qk_rope_reshape_and_cache``)
  is not installed here; this restatement defines its cache value as what the
  unfused sequence (rotation, then ``reshape_and_cache_flash``) stores: the
  rotated key rounded to the model dtype, then quantised.

fp32 arithmetic is numpy's (IEEE, round to nearest); float -> fp8 is the own
encoder :func:`fp8_encode` (round to nearest even, saturating at the largest
finite value, as a ``cvt.rn.satfinite`` conversion does).
"""

from __future__ import annotations

import numpy as np
import torch

from .rope import reference_rope

# name -> (mantissa bits, exponent bias, largest finite value, NaN code)
FP8_FORMATS = {
    "e4m3": (3, 7, 448.0, 0x7F),
    "e5m2": (2, 15, 57344.0, 0x7F),
}
QUANT_RANGES = {"int8": (127.0, -128.0), "e4m3": (448.0, -448.0)}


def fp8_encode(x: np.ndarray, fmt: str = "e4m3") -> np.ndarray:
    """float32 values -> fp8 codes (uint8): round to nearest even, saturate to +-max finite."""
    man, bias, max_finite, nan_code = FP8_FORMATS[fmt]
    with np.errstate(invalid="ignore"):  # signalling-NaN inputs
        x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = np.signbit(x)
    nan = np.isnan(x)
    a = np.minimum(np.abs(np.where(nan, 0.0, x)), max_finite)
    min_exp = 1 - bias
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    quantum = np.exp2(np.maximum(e, min_exp) - man)
    q = np.minimum(np.round(a / quantum) * quantum, max_finite)  # np.round: half to even
    eq = np.floor(np.log2(np.where(q > 0, q, 1.0)))
    normal = (q > 0) & (eq >= min_exp)
    exp_field = np.where(normal, eq + bias, 0)
    mant = np.where(normal, q / np.exp2(eq - man) - 2**man, q / 2.0 ** (min_exp - man))
    code = (exp_field.astype(np.int64) << man) | np.rint(mant).astype(np.int64)
    code = np.where(sign, code | 0x80, code)
    code = np.where(nan, nan_code, code)
    return code.astype(np.uint8)


def fp8_decode(code: np.ndarray, fmt: str = "e4m3") -> np.ndarray:
    """fp8 codes -> float32 (NaN codes -> NaN)."""
    man, bias, _, _ = FP8_FORMATS[fmt]
    c = np.asarray(code, dtype=np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    ef = (c >> man) & ((0x7F >> man))
    mf = c & ((1 << man) - 1)
    val = np.where(ef == 0, mf * 2.0 ** (1 - bias - man), (1 + mf / 2.0**man) * np.exp2(ef - bias))
    out = sign * val
    if fmt == "e4m3":
        out = np.where((c & 0x7F) == 0x7F, np.nan, out)
    else:
        out = np.where((ef == 0x1F) & (mf != 0), np.nan, np.where(ef == 0x1F, sign * np.inf, out))
    return out.astype(np.float32)


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy()


def quantize_per_tensor(x: torch.Tensor, scale: float, fmt: str = "e4m3") -> np.ndarray:
    """``fp8(x / scale)``: the quotient in fp32 (round to nearest), then :func:`fp8_encode`."""
    return fp8_encode(_f32(x) / np.float32(scale), fmt)


def quantize_per_token_head(x: torch.Tensor, kind: str) -> tuple[np.ndarray, np.ndarray]:
    """Rows ``x [..., D]`` -> (codes [..., D] as int8 / fp8 codes, scales [...] float32)."""
    qmax, qmin = QUANT_RANGES[kind]
    xf = _f32(x)
    amax = np.abs(xf).max(axis=-1)
    s = np.maximum(amax / np.float32(qmax), np.float32(1e-6)).astype(np.float32)
    inv = (np.float32(1.0) / s).astype(np.float32)
    q = np.clip(xf * inv[..., None], np.float32(qmin), np.float32(qmax)).astype(np.float32)
    if kind == "int8":
        return np.trunc(q).astype(np.int8), s
    return fp8_encode(q, "e4m3"), s


def kv_write_reference(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    kv_cache_dtype: str,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
    k_scale_cache: torch.Tensor | None = None,
    v_scale_cache: torch.Tensor | None = None,
):
    """Expected caches (and scale caches) after the service's cache update.

    ``key_cache``/``value_cache`` are ``[num_blocks, block_size, KH, >= D]``
    CPU tensors (copied, not modified); fp8 caches are returned as uint8 code
    tensors, int8 caches as int8.  Returns ``(kc, vc, ksc, vsc)``; the scale
    caches are ``None`` except in the per-token-head modes.
    """
    d = key.shape[2]
    fp8_cache = key_cache.dtype in (torch.float8_e4m3fn, torch.float8_e5m2)
    kc = key_cache.detach().cpu().clone()
    vc = value_cache.detach().cpu().clone()
    if fp8_cache:
        kc, vc = kc.view(torch.uint8), vc.view(torch.uint8)
    ksc = k_scale_cache.detach().cpu().clone() if k_scale_cache is not None else None
    vsc = v_scale_cache.detach().cpu().clone() if v_scale_cache is not None else None
    slots = slot_mapping.cpu().long()
    idx = torch.nonzero(slots >= 0).flatten()
    bs = kc.shape[1]
    blocks = torch.div(slots[idx], bs, rounding_mode="floor")
    offs = slots[idx] - blocks * bs
    k_rows, v_rows = key.detach().cpu()[idx], value.detach().cpu()[idx]
    if kv_cache_dtype == "auto":
        kc[blocks, offs, :, :d] = k_rows.to(kc.dtype)
        vc[blocks, offs, :, :d] = v_rows.to(vc.dtype)
    elif kv_cache_dtype.endswith("per_token_head"):
        kind = "int8" if kv_cache_dtype.startswith("int8") else "e4m3"
        for rows, cache, sc in ((k_rows, kc, ksc), (v_rows, vc, vsc)):
            codes, s = quantize_per_token_head(rows, kind)
            cache[blocks, offs, :, :d] = torch.from_numpy(codes)
            sc[blocks, offs] = torch.from_numpy(s)
    else:  # fp8 per-tensor, written as e4m3 whatever the storage dtype
        kc[blocks, offs, :, :d] = torch.from_numpy(quantize_per_tensor(k_rows, k_scale))
        vc[blocks, offs, :, :d] = torch.from_numpy(quantize_per_tensor(v_rows, v_scale))
    return kc, vc, ksc, vsc


def dequantize_cache_reference(cache_codes: torch.Tensor, kv_cache_dtype: str, head_dim: int,
                               scale: float | None = None, scale_cache: torch.Tensor | None = None) -> torch.Tensor:
    """The values vLLM's unified attention reads from a quantised cache, in fp32.

    Follows vLLM 0.22 ``vllm/v1/attention/ops/triton_unified_attention.py``:
    fp8 per-tensor (``_cast_kv_tile``, :39-55): ``fp8(x) * scale``; int8 / fp8
    per-token-head (:469-511): the element times the scale of its (block,
    slot, head), which vLLM folds into the logits (keys) and into P (values).
    ``cache_codes [num_blocks, block_size, KH, >= head_dim]``: int8 values or
    fp8 codes (uint8 / float8 storage).  Returns ``[num_blocks, block_size, KH,
    head_dim]`` float32.
    """
    c = cache_codes.detach().cpu()[..., :head_dim]
    if kv_cache_dtype.endswith("per_token_head"):
        if kv_cache_dtype.startswith("int8"):
            vals = c.view(torch.int8).float().numpy()
        else:
            vals = fp8_decode(c.contiguous().view(torch.uint8).numpy(), "e4m3")
        s = scale_cache.detach().cpu().float().numpy()[..., None]
        return torch.from_numpy((vals * s).astype(np.float32))
    fmt = "e5m2" if kv_cache_dtype == "fp8_e5m2" else "e4m3"
    vals = fp8_decode(c.contiguous().view(torch.uint8).numpy(), fmt)
    return torch.from_numpy((vals * np.float32(scale)).astype(np.float32))


def rope_and_cache_service_reference(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    is_neox: bool,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: float,
    v_scale: float,
    apply_scale: bool,
):
    """Expected ``(query, key, key_cache, value_cache)`` after the service's rope-and-cache call."""
    rd = int(cos_sin_cache.shape[1])
    q_out = reference_rope(query, cos_sin_cache, positions, is_neox, rd)
    k_out = reference_rope(key, cos_sin_cache, positions, is_neox, rd)
    kc, vc, _, _ = kv_write_reference(
        k_out, value, key_cache, value_cache, slot_mapping, "fp8" if apply_scale else "auto", k_scale, v_scale
    )
    return q_out, k_out, kc, vc
