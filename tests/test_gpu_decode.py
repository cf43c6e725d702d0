"""Parity of the sm_100a decode kernel (batches with one query token per sequence).

A batch whose ``max_seqlen_q`` is 1 runs the persistent decode kernel and its
combine (the operator API is unchanged).  Bar: the same bf16 tolerances as the
prefill path against the fp32 oracle, on key lengths around page, tile and
chunk boundaries, empty sequences, NaN garbage past the sequence end, GQA
ratios 4 / 8 / 16, fp16, int64 indices, the 16K decode workload in full, and
agreement with the prefill kernel on the same batch.
"""

from __future__ import annotations

import pytest
import torch

from helpers import assert_close, oracle, run_gpu
from minicpm_b200 import _lib, iluvatar_attention
from minicpm_b200.workloads import build_attention_batch, lengths_decode_4k, lengths_decode_16k

pytestmark = pytest.mark.gpu


def _no_device_error():
    assert _lib.device_error() == _lib.DEVERR_NONE


def _decode_batch(kv_lens, **kw):
    return build_attention_batch([1] * len(kv_lens), kv_lens, **kw)


EDGE_LENGTHS = [1, 2, 15, 16, 17, 127, 128, 129, 255, 256, 257, 1000, 1024, 3001, 4096, 4097, 8191]


def test_edge_lengths():
    batch = _decode_batch(EDGE_LENGTHS, seed=21, pool_pages=2000)
    want = oracle(batch)
    for s in (0, 1, 4):  # the split count does not change the decode path
        assert_close(run_gpu(batch, s), want, f"decode edges S={s}")
    _no_device_error()


def test_more_sequences_than_the_schedule_caches():
    """5000 decode rows: past the decode schedule's shared-memory copy of the
    item prefix (4096 sequences), so it searches the workspace array; every
    97th row and the last ones against the oracle."""
    n = 5000
    kv = [1 + (i * 37) % 700 for i in range(n)]
    kv[17] = 9000  # one long row among the short ones
    batch = _decode_batch(kv, seed=5000)
    got = run_gpu(batch, 0)
    picks = list(range(0, n, 97)) + [17, n - 2, n - 1]
    sub = build_attention_batch([1] * len(picks), [kv[i] for i in picks], seed=5000, seq_ids=picks)
    # content is keyed on the sequence ids, so the sub-batch holds the same rows
    assert torch.equal(sub.q, batch.q[picks])
    assert_close(got[picks], oracle(sub), "5000 decode rows")
    _no_device_error()


def test_matches_prefill_kernel(monkeypatch):
    batch = _decode_batch([333, 4096, 70, 12000, 1, 640], seed=22)
    got = run_gpu(batch, 0)
    monkeypatch.setenv("B200_ATTN_DECODE", "0")
    ref = run_gpu(batch, 0)
    assert_close(got, ref, "decode vs prefill kernel", atol_max=1.6e-2, atol_mean=1e-3)
    assert_close(got, oracle(batch), "decode vs oracle")


def test_empty_sequences_and_zero_keys():
    # Sequence 1 has no query token (no output row), sequence 2 has one token
    # but no key (its row is 0), the rest are ordinary.
    batch = build_attention_batch([1, 0, 1, 1], [50, 30, 0, 700], seed=23)
    want = oracle(batch)
    got = run_gpu(batch, 0)
    assert_close(got, want, "decode empty")
    assert got[1].abs().max().item() == 0.0
    _no_device_error()


def test_nan_past_the_sequence_end_is_ignored():
    batch = _decode_batch([20, 131, 16, 250], seed=24, pool_pages=64)
    want = oracle(batch)
    cache = batch.kv_cache.clone()
    for row, L in enumerate(batch.kv_lens):
        if L % 16:
            last = int(batch.block_table[row, (L - 1) // 16])
            cache[last, :, L % 16 :] = float("nan")
    used = set(batch.block_table.flatten().tolist())
    for p in range(cache.shape[0]):
        if p not in used:
            cache[p] = float("nan")
    batch.kv_cache = cache
    assert_close(run_gpu(batch, 0), want, "decode nan tail")


@pytest.mark.parametrize("hq,hkv", [(8, 2), (16, 2), (16, 1), (32, 8)])
def test_gqa_ratios(hq, hkv):
    batch = _decode_batch([77, 1500, 260, 5000], seed=25, num_q_heads=hq, num_kv_heads=hkv)
    assert_close(run_gpu(batch, 0), oracle(batch), f"decode hq={hq} hkv={hkv}")
    _no_device_error()


def test_fp16_and_int64_indices():
    batch = _decode_batch([900, 33, 2048], seed=26, dtype=torch.float16)
    b = batch.to("cuda")
    out = torch.empty_like(b.q)
    from minicpm_b200 import paged_split_kv_attention

    paged_split_kv_attention(
        b.q, b.kv_cache[:, 0], b.kv_cache[:, 1], out, b.block_table.long(), b.seqused_k.long(), b.cu_seqlens_q.long(),
        1, b.max_seqlen_k, b.softmax_scale, num_splits=0,
    )
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    assert_close(out.cpu(), oracle(batch), "decode fp16 int64")


def test_mislabelled_batch_is_reported():
    # max_seqlen_q = 1 while sequence 0 holds two query tokens: the decode
    # schedule records it (that sequence's rows are left as they were).
    batch = build_attention_batch([2, 1], [40, 90], seed=27)
    b = batch.to("cuda")
    out = torch.zeros_like(b.q)
    from minicpm_b200 import paged_split_kv_attention

    paged_split_kv_attention(b.q, b.kv_cache[:, 0], b.kv_cache[:, 1], out, b.block_table, b.seqused_k,
                             b.cu_seqlens_q, 1, b.max_seqlen_k, b.softmax_scale)
    assert _lib.device_error() == _lib.DEVERR_DECODE_QLEN
    want = oracle(batch)
    assert_close(out[2:3].cpu(), want[2:3], "decode mislabelled, well-formed row")


@pytest.mark.parametrize("lengths", [lengths_decode_16k, lengths_decode_4k])
def test_full_decode_workloads(lengths):
    q, kv = lengths()
    batch = build_attention_batch(q, kv)
    assert_close(run_gpu(batch, 0), oracle(batch), lengths.__name__)
    _no_device_error()


def test_dispatcher_routes_decode_only_when_enabled(monkeypatch):
    batch = _decode_batch([100, 900], seed=28)
    b = batch.to("cuda")
    out = torch.empty_like(b.q)
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV_DECODE", "1")
    iluvatar_attention(b.q, b.kv_cache, b.kv_cache, out, b.cu_seqlens_q, 1, b.seqused_k, b.max_seqlen_k,
                       b.softmax_scale, causal=True, block_table=b.block_table)
    torch.cuda.synchronize()
    assert_close(out.cpu(), oracle(batch), "dispatcher decode")
