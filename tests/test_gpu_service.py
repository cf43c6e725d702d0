"""The service shim end to end on the GPU: cache update, then attention, as a serving step runs them.

A step's new K/V rows are removed from the paged cache, written back through
``do_kv_cache_update`` (or the fused ``do_rope_and_kv_cache_update``), and
``forward`` then attends over the cache; the result must match the fp32 oracle
of the original batch.  The sm_100a route is checked to be the one taken
(prefill with the two enable flags; decode with the decode flag), and the
decode step without the flag is checked on vLLM's own kernel where vLLM runs.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from helpers import assert_close, oracle
from minicpm_b200 import _lib, service
from minicpm_b200.workloads import build_attention_batch, build_rope_batch
from oracle import rope_and_cache_service_reference

pytestmark = pytest.mark.gpu


def _enable(monkeypatch, decode=False):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    if decode:
        monkeypatch.setenv("ILUVATAR_SPLIT_KV_DECODE", "1")
    else:
        monkeypatch.delenv("ILUVATAR_SPLIT_KV_DECODE", raising=False)


def _spy(monkeypatch):
    calls = []
    real = service.unified_attention_optimized

    def wrapped(**kw):
        calls.append(kw["max_seqlen_q"])
        return real(**kw)

    monkeypatch.setattr(service, "unified_attention_optimized", wrapped)
    return calls


def _step(batch):
    """Slots of the step's new tokens, their K/V rows, and the cache with those rows zeroed."""
    slots, rows = [], []
    for b, (q, L) in enumerate(zip(batch.query_lens, batch.kv_lens)):
        for i in range(q):
            p = L - q + i
            blk = int(batch.block_table[b, p // 16])
            slots.append(blk * 16 + p % 16)
            rows.append((blk, p % 16))
    slot_mapping = torch.tensor(slots, dtype=torch.int64)
    blk = torch.tensor([r[0] for r in rows])
    off = torch.tensor([r[1] for r in rows])
    key = batch.kv_cache[blk, 0, off].clone()
    value = batch.kv_cache[blk, 1, off].clone()
    cache = batch.kv_cache.clone()
    cache[blk, :, off] = 0
    return key, value, slot_mapping, cache


def _metadata(batch, device):
    g = batch.to(device)
    builder = service.IluvatarAttentionMetadataBuilder(batch.q.shape[1], batch.kv_cache.shape[3], batch.q.shape[2], device)
    common = SimpleNamespace(
        num_reqs=len(batch.query_lens), num_actual_tokens=batch.total_q, max_query_len=batch.max_seqlen_q,
        max_seq_len=batch.max_seqlen_k, query_start_loc=g.cu_seqlens_q, seq_lens=g.seqused_k,
        block_table_tensor=g.block_table, slot_mapping=None, causal=True,
    )
    return builder.build(0, common)


def _layer():
    one = torch.tensor(1.0, device="cuda")
    return SimpleNamespace(_k_scale=one, _v_scale=one, _q_scale=one)


def _serve(batch, decode_flag, monkeypatch):
    key, value, slot_mapping, cache = _step(batch)
    dev = torch.device("cuda")
    kv_cache = cache.to(dev)
    impl = service.IluvatarAttentionImpl(batch.q.shape[1], batch.q.shape[2], batch.softmax_scale, kv_cache.shape[3],
                                         None, None, "auto")
    impl.do_kv_cache_update(_layer(), key.to(dev), value.to(dev), kv_cache, slot_mapping.to(dev))
    meta = _metadata(batch, dev)
    q = batch.q.to(dev)
    out = torch.empty_like(q)
    impl.forward(_layer(), q, q, q, kv_cache, meta, out)
    torch.cuda.synchronize()
    assert torch.equal(kv_cache.cpu(), batch.kv_cache), "cache update restored the step's rows"
    return out.cpu()


def test_prefill_step_takes_the_b200_route(monkeypatch):
    _enable(monkeypatch)
    calls = _spy(monkeypatch)
    batch = build_attention_batch([37, 128, 5, 300], [37, 700, 900, 2000], seed=31)
    got = _serve(batch, False, monkeypatch)
    assert calls == [batch.max_seqlen_q]
    assert_close(got, oracle(batch), "service prefill")
    assert _lib.device_error() == _lib.DEVERR_NONE


def test_decode_step_with_the_decode_flag(monkeypatch):
    _enable(monkeypatch, decode=True)
    calls = _spy(monkeypatch)
    batch = build_attention_batch([1] * 6, [5, 130, 1000, 4097, 77, 2048], seed=32)
    got = _serve(batch, True, monkeypatch)
    assert calls == [1]
    assert_close(got, oracle(batch), "service decode")


def test_decode_step_without_the_flag_stays_on_vllm(monkeypatch):
    try:
        from vllm.v1.attention.ops.triton_unified_attention import unified_attention  # noqa: F401
    except Exception as exc:
        pytest.skip(f"vLLM not importable: {exc}")
    _enable(monkeypatch, decode=False)
    calls = _spy(monkeypatch)
    batch = build_attention_batch([1] * 4, [17, 300, 1024, 33], seed=33)
    try:
        got = _serve(batch, False, monkeypatch)
    except Exception as exc:  # pragma: no cover - vLLM's kernel on this box
        pytest.skip(f"vLLM's unified_attention did not run here: {exc}")
    assert calls == []
    assert_close(got, oracle(batch), "vLLM decode")


@pytest.mark.parametrize("fp8", [False, True])
def test_rope_and_cache_update_hook(fp8):
    b = build_rope_batch(512, rotary_dim=128, is_neox=True, num_blocks=64)
    dev = torch.device("cuda")
    g = b.to(dev)
    nb, bs, kh, d = b.key_cache.shape
    dtype = torch.uint8 if fp8 else torch.bfloat16
    kv_cache = torch.zeros(nb, 2, bs, kh, d, dtype=dtype, device=dev)
    impl = service.IluvatarAttentionImpl(16, 128, 0.088, kh, None, None, "fp8" if fp8 else "auto")
    assert impl.fused_rope_kvcache_supported()
    layer = SimpleNamespace(_k_scale=torch.tensor([0.02], device=dev), _v_scale=torch.tensor([0.03], device=dev))
    impl.do_rope_and_kv_cache_update(layer, g.query, g.key, g.value, g.positions, g.cos_sin_cache, True, kv_cache,
                                     g.slot_mapping)
    torch.cuda.synchronize()
    kc0 = torch.zeros(nb, bs, kh, d, dtype=dtype)
    if fp8:
        kc0 = kc0.view(torch.float8_e4m3fn)
    q_want, k_want, kc_want, vc_want = rope_and_cache_service_reference(
        b.query, b.key, b.value, b.positions, b.cos_sin_cache, True, kc0, kc0.clone(), b.slot_mapping, 0.02, 0.03, fp8
    )
    u8 = lambda t: t.detach().cpu().contiguous().view(torch.uint8)  # noqa: E731
    assert torch.equal(u8(g.query), u8(q_want)) and torch.equal(u8(g.key), u8(k_want))
    assert torch.equal(u8(kv_cache[:, 0]), u8(kc_want)) and torch.equal(u8(kv_cache[:, 1]), u8(vc_want))
