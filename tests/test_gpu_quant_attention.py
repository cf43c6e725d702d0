"""Attention over quantised KV caches on the GPU, against the oracle.

The reference's service sends these calls to vLLM's unified_attention
(integration/vllm-plugin-FL-split-kv.patch:473-523); here the pages a call
references are dequantised (``b200_kv_dequant_pages``) and the sm_100a
attention kernel runs on them.  The oracle dequantises the same cache codes
in fp32 (``oracle.dequantize_cache_reference``, vLLM's arithmetic) and runs
the fp32 paged attention; the tolerance is the bf16 attention tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close, small_batch
from minicpm_b200 import _lib, iluvatar_attention
from minicpm_b200.workloads import KvWriteBatch
from oracle import dequantize_cache_reference, paged_attention_reference, quantize_per_tensor, quantize_per_token_head

pytestmark = pytest.mark.gpu

MODES = {"fp8": 1, "fp8_e5m2": 1, "int8_per_token_head": 2, "fp8_per_token_head": 3}
TORCH_FP8 = {"fp8": torch.float8_e4m3fn, "fp8_e5m2": torch.float8_e5m2}


def _inline_scale_views(cache, kh, d, kind):
    """Float views of the scales stored after head_dim in each row of a 5-D cache (the service's layout)."""
    kb = KvWriteBatch(key=torch.empty(1, kh, d, device=cache.device), value=None, slot_mapping=None, kv_cache=cache,
                      kv_cache_dtype=kind, k_scale=None, v_scale=None)
    return kb.scale_cache_views()


def _quantised(batch, kind, inline):
    """Cache codes and scales for every page of ``batch``'s pool, in the layout the service uses
    (per-token-head scales inline after head_dim when ``inline``)."""
    k_all, v_all = batch.kv_cache[:, 0], batch.kv_cache[:, 1]
    nb, bs, kh, d = k_all.shape
    if MODES[kind] == 1:
        fmt = "e5m2" if kind == "fp8_e5m2" else "e4m3"
        ks, vs = 0.0125, 0.0089
        kc = torch.from_numpy(quantize_per_tensor(k_all, ks, fmt)).view(TORCH_FP8[kind])
        vc = torch.from_numpy(quantize_per_tensor(v_all, vs, fmt)).view(TORCH_FP8[kind])
        want_k = dequantize_cache_reference(kc.view(torch.uint8), kind, d, scale=ks)
        want_v = dequantize_cache_reference(vc.view(torch.uint8), kind, d, scale=vs)
        return dict(kc=kc, vc=vc, k_descale=torch.full((1, kh), ks), v_descale=torch.full((1, kh), vs)), want_k, want_v
    qkind = "int8" if kind.startswith("int8") else "e4m3"
    k_codes, k_s = quantize_per_token_head(k_all, qkind)
    v_codes, v_s = quantize_per_token_head(v_all, qkind)
    dt = torch.int8 if qkind == "int8" else torch.float8_e4m3fn
    if inline:
        cache = torch.zeros(nb, 2, bs, kh, d + 4, dtype=torch.uint8)
        cache[:, 0, ..., :d] = torch.from_numpy(k_codes).view(torch.uint8)
        cache[:, 1, ..., :d] = torch.from_numpy(v_codes).view(torch.uint8)
        ksv, vsv = _inline_scale_views(cache, kh, d, kind)
        ksv.copy_(torch.from_numpy(k_s))
        vsv.copy_(torch.from_numpy(v_s))
        kc, vc = cache.view(dt).unbind(1)
        extra = dict(cache=cache)
    else:
        kc, vc = torch.from_numpy(k_codes).view(dt), torch.from_numpy(v_codes).view(dt)
        ksv, vsv = torch.from_numpy(k_s), torch.from_numpy(v_s)
        extra = {}
    want_k = dequantize_cache_reference(kc.view(torch.uint8) if dt != torch.int8 else kc, kind, d, scale_cache=ksv)
    want_v = dequantize_cache_reference(vc.view(torch.uint8) if dt != torch.int8 else vc, kind, d, scale_cache=vsv)
    return dict(kc=kc, vc=vc, k_scale_cache=ksv, v_scale_cache=vsv, **extra), want_k, want_v


@pytest.mark.parametrize("kind", list(MODES))
@pytest.mark.parametrize("inline", [False, True])
def test_attention_over_quantised_cache(monkeypatch, kind, inline):
    if inline and MODES[kind] == 1:
        pytest.skip("per-tensor caches carry no inline scale")
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    batch = small_batch([37, 1, 100, 300], [200, 63, 1000, 2500], seed=77, pool_pages=400)
    parts, want_k, want_v = _quantised(batch, kind, inline)
    want = paged_attention_reference(batch.q, want_k, want_v, batch.block_table, batch.cu_seqlens_q, batch.seqused_k,
                                     batch.softmax_scale)
    dev = torch.device("cuda")
    q = batch.q.to(dev)
    if "cache" in parts:  # the service's 5-D layout, views into one buffer
        cache = parts["cache"].to(dev)
        ksc, vsc = _inline_scale_views(cache, cache.shape[3], cache.shape[4] - 4, kind)
        dt = torch.int8 if kind.startswith("int8") else torch.float8_e4m3fn
        kc, vc = cache.view(dt).unbind(1)
    else:
        kc, vc = parts["kc"].to(dev), parts["vc"].to(dev)
        ksc = parts.get("k_scale_cache")
        vsc = parts.get("v_scale_cache")
        ksc = ksc.to(dev) if ksc is not None else None
        vsc = vsc.to(dev) if vsc is not None else None
    kdes = parts.get("k_descale")
    vdes = parts.get("v_descale")
    for splits in ("1", "4"):
        monkeypatch.setenv("ILUVATAR_NUM_SPLITS", splits)
        out = torch.full_like(q, float("nan"))
        iluvatar_attention(q, kc, vc, out, batch.cu_seqlens_q.to(dev), batch.max_seqlen_q, batch.seqused_k.to(dev),
                           batch.max_seqlen_k, batch.softmax_scale, causal=True, block_table=batch.block_table.to(dev),
                           kv_quant_mode=MODES[kind],
                           k_descale=kdes.to(dev) if kdes is not None else None,
                           v_descale=vdes.to(dev) if vdes is not None else None,
                           k_scale_cache=ksc, v_scale_cache=vsc)
        torch.cuda.synchronize()
        assert_close(out.cpu(), want, f"{kind} inline={inline} S={splits}")
    assert _lib.device_error() == _lib.DEVERR_NONE


def test_dequantised_pages_match_the_oracle_exactly_in_bf16():
    """The dense pages themselves: every referenced page equals the oracle's
    fp32 dequantisation rounded to bf16; the dense block table is b * max_pages + p."""
    from minicpm_b200.kv_cache import dequantize_kv_pages

    batch = small_batch([5, 9], [300, 40], seed=78, pool_pages=64)
    parts, want_k, want_v = _quantised(batch, "int8_per_token_head", inline=False)
    dev = torch.device("cuda")
    cache, table = dequantize_kv_pages(parts["kc"].to(dev), parts["vc"].to(dev), batch.block_table.to(dev),
                                       batch.seqused_k.to(dev), batch.max_seqlen_k, 2, torch.bfloat16, 128,
                                       k_scale_cache=parts["k_scale_cache"].to(dev),
                                       v_scale_cache=parts["v_scale_cache"].to(dev))
    torch.cuda.synchronize()
    max_pages = -(-batch.max_seqlen_k // 16)
    assert torch.equal(table.cpu(), torch.arange(2 * max_pages, dtype=torch.int32).view(2, max_pages))
    got = cache.cpu()
    for b, L in enumerate(batch.kv_lens):
        for p in range(-(-L // 16)):
            src = int(batch.block_table[b, p])
            assert torch.equal(got[b * max_pages + p, 0], want_k[src].to(torch.bfloat16))
            assert torch.equal(got[b * max_pages + p, 1], want_v[src].to(torch.bfloat16))
