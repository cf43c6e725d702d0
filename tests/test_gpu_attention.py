"""Parity of the sm_100a paged attention against the fp32 oracle (GPU).

Cases follow the reference's own unit test (tests/test_paged_split_kv.py:105-114:
three shape sets x splits 4 and 8, permuted block table) plus the edge cases
of its semantics: partial last pages, rows whose split holds no key, decode
rows (q_len = 1), empty requests, seqused_k < q_len, int64 indices, fp16,
other GQA ratios, page size 32, strided q, and NaN garbage in page tails.
"""

from __future__ import annotations

import math

import pytest
import torch

from helpers import (ATOL_MAX, ATOL_MEAN, assert_close, errors, oracle, run_gpu, sample_blocks, sampled_oracle,
                     small_batch)
from minicpm_b200 import _lib, iluvatar_attention, paged_split_kv_attention, split_kv_combine
from minicpm_b200.workloads import (build_attention_batch, correctness_batch, lengths_chunked_4k, lengths_chunked_16k,
                                    lengths_mixed)

pytestmark = pytest.mark.gpu

REFERENCE_CASES = [
    ([1, 17, 65], [127, 111, 63]),
    ([31, 1, 13], [0, 255, 1001]),
    ([64, 1, 1], [2048, 4096, 8192]),
]


def _no_device_error():
    assert _lib.device_error() == _lib.DEVERR_NONE


@pytest.mark.parametrize("case", range(3))
@pytest.mark.parametrize("splits", [4, 8, 1, 0])
def test_reference_unit_cases(case, splits):
    ql, pre = REFERENCE_CASES[case]
    batch = small_batch(ql, pre, seed=20260928 + case)
    got = run_gpu(batch, splits)
    assert_close(got, oracle(batch).to(torch.bfloat16), f"case{case} S={splits}")
    _no_device_error()


@pytest.mark.parametrize("splits", [1, 2, 4, 8, 16, 0])
def test_correctness_config(splits):
    batch = correctness_batch()
    got = run_gpu(batch, splits)
    assert_close(got, oracle(batch), f"correctness S={splits}")
    _no_device_error()


def test_edge_lengths():
    # KV lengths around page and tile boundaries, decode rows, a 1-token
    # sequence, and query chunks that end mid-tile.
    ql = [1, 1, 2, 15, 16, 17, 127, 128, 129, 1, 300]
    pre = [0, 15, 14, 1, 0, 111, 1, 128, 127, 4095, 17]
    batch = small_batch(ql, pre, seed=7, pool_pages=400)
    want = oracle(batch)
    for s in (1, 2, 4, 16):
        assert_close(run_gpu(batch, s), want, f"edges S={s}")
    _no_device_error()


def test_empty_request_and_no_key_rows():
    # Request 1 has no query rows; request 2 has seqused_k < q_len so its
    # first rows see no key (they are 0, as the kernel's acc / max(l, 1e-20)).
    batch = build_attention_batch([5, 0, 20], [40, 10, 12], seed=3)
    want = oracle(batch)
    for s in (1, 4):
        got = run_gpu(batch, s)
        assert_close(got, want, f"empty/no-key S={s}")
        assert got[5:13].abs().max().item() == 0.0
    _no_device_error()


def test_nan_in_page_tail_is_ignored():
    batch = small_batch([9, 30], [20, 3], seed=11, pool_pages=8)
    want = oracle(batch)
    cache = batch.kv_cache.clone()
    for row, L in enumerate(batch.kv_lens):
        last = int(batch.block_table[row, (L - 1) // 16])
        cache[last, :, L % 16 :] = float("nan")
        # Pages that belong to nobody hold NaN too.
    used = set(batch.block_table.flatten().tolist())
    for p in range(cache.shape[0]):
        if p not in used:
            cache[p] = float("nan")
    batch.kv_cache = cache
    for s in (1, 2):
        assert_close(run_gpu(batch, s), want, f"nan tail S={s}")


def test_int64_indices_and_wide_table():
    batch = small_batch([33, 7], [100, 500], seed=5, extra_table_cols=9)
    want = oracle(batch)
    b = batch.to("cuda")
    out = torch.empty_like(b.q)
    paged_split_kv_attention(
        b.q, b.kv_cache[:, 0], b.kv_cache[:, 1], out, b.block_table.long(), b.seqused_k.long(), b.cu_seqlens_q.long(),
        b.max_seqlen_q, b.max_seqlen_k, b.softmax_scale, num_splits=2,
    )
    assert_close(out.cpu(), want, "int64")


def test_fp16():
    batch = small_batch([40, 3], [200, 77], seed=9, dtype=torch.float16)
    got = run_gpu(batch, 1)
    assert got.dtype == torch.float16
    assert_close(got, oracle(batch), "fp16")


@pytest.mark.parametrize("hq,hkv", [(8, 1), (16, 16), (32, 2), (4, 2), (12, 2), (6, 2), (40, 4), (80, 1), (128, 1)])
def test_other_gqa_ratios(hq, hkv):
    """Ratios that divide 128 and ratios that do not (6:1, 3:1, 10:1, 80:1: a
    query tile holds floor(128 / G) positions x G heads, the rest is padding)."""
    batch = small_batch([19, 70], [45, 300], seed=13, num_q_heads=hq, num_kv_heads=hkv)
    for s in (1, 4):
        assert_close(run_gpu(batch, s), oracle(batch), f"gqa {hq}/{hkv} S={s}")


def test_page_size_32():
    batch = small_batch([50, 9], [77, 400], seed=17, block_size=32)
    assert_close(run_gpu(batch, 2), oracle(batch), "bs32")


def test_strided_query_and_5d_cache_through_dispatcher(monkeypatch):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    monkeypatch.setenv("ILUVATAR_NUM_SPLITS", "4")
    batch = small_batch([21, 40], [10, 200], seed=19)
    want = oracle(batch)
    b = batch.to("cuda")
    # q as a view into a wider [T, H + 2*KH, D] qkv buffer.
    qkv = torch.randn(b.q.shape[0], 16 + 4, 128, device="cuda", dtype=torch.bfloat16)
    qkv[:, :16] = b.q
    q = qkv[:, :16]
    out = torch.empty(b.q.shape, device="cuda", dtype=torch.bfloat16)
    ret = iluvatar_attention(
        q, b.kv_cache, b.kv_cache, out, b.cu_seqlens_q, b.max_seqlen_q, b.seqused_k, b.max_seqlen_k,
        b.softmax_scale, causal=True, block_table=b.block_table,
    )
    assert ret is out
    assert_close(out.cpu(), want, "dispatcher 5-D cache")


def test_zero_lengths_return_zeros():
    batch = small_batch([4], [4], seed=1).to("cuda")
    out = torch.full_like(batch.q, 3.0)
    ret = paged_split_kv_attention(
        batch.q, batch.kv_cache[:, 0], batch.kv_cache[:, 1], out, batch.block_table, batch.seqused_k,
        batch.cu_seqlens_q, 0, batch.max_seqlen_k, batch.softmax_scale,
    )
    assert ret is out and out.abs().max().item() == 0.0


def test_deterministic_and_page_permutation_invariant():
    q, kv = lengths_chunked_4k(num_seqs=6)
    batch = build_attention_batch(q, kv, seed=23)
    a = run_gpu(batch, 1)
    b = run_gpu(batch, 1)
    assert torch.equal(a, b)
    # Move every page to a new physical slot: the output must not change at all.
    perm = torch.randperm(batch.kv_cache.shape[0], generator=torch.Generator().manual_seed(5))
    moved = batch.kv_cache.clone()
    moved[perm] = batch.kv_cache
    batch2 = build_attention_batch(q, kv, seed=23)
    batch2.kv_cache = moved
    batch2.block_table = perm[batch.block_table.long()].to(torch.int32)
    assert torch.equal(run_gpu(batch2, 1), a)


def test_chunked_prefill_4k_full_config_against_oracle():
    """The whole 4K config (64 sequences, 512-token chunks, KV 1024-4096) at
    S = 4 and 8 (the reference test's split counts,
    tests/test_paged_split_kv.py:105-114) and auto: the first, middle and last
    16 rows of every sequence against the oracle."""
    q, kv = lengths_chunked_4k()
    batch = build_attention_batch(q, kv)
    want, rows = sampled_oracle(batch, sample_blocks(q))
    for s in (4, 8, 0):
        assert_close(run_gpu(batch, s)[rows], want, f"4k S={s}")
    _no_device_error()


def _split_slots() -> int:
    """Split-unit slots the last call's schedule kernel made (its workspace counter)."""
    dev = torch.cuda.current_device()
    ws = _lib._workspaces[(dev, torch.cuda.current_stream().cuda_stream)]
    return int(ws[:12].cpu().view(torch.int32)[2])


def test_schedule_beyond_its_shared_memory_caches(monkeypatch):
    """9000 sequences and 9015 query units: more than the schedule kernel keeps
    in shared memory (4096 sequences, 8192 query units), so every pass reads
    the workspace arrays instead; two long sequences among the short ones.
    Sampled sequences against the oracle at S = auto / 4 and every unit split
    4 ways."""
    n = 9000
    q = [2] * n
    kv = [40 + (i % 7) * 9 for i in range(n)]
    q[5], kv[5] = 300, 5000
    q[4000], kv[4000] = 200, 3000
    batch = build_attention_batch(q, kv, seed=9000)
    picks = [(s, 0, q[s]) for s in range(0, n, 97)] + [(5, 0, 300), (4000, 0, 200), (n - 1, 0, 2)]
    want, rows = sampled_oracle(batch, picks)
    for s in (0, 4):
        assert_close(run_gpu(batch, s)[rows], want, f"9000 seqs S={s}")
    monkeypatch.setenv("B200_ATTN_SPLIT_UNIFORM", "1")
    assert_close(run_gpu(batch, 4)[rows], want, "9000 seqs uniform S=4")
    _no_device_error()


def test_split_policy_splits_small_batches_only():
    """num_splits is the most any query unit gets: the reference's third unit
    case (few sequences, long keys) is split, the 4K config (13 waves of units
    on 148 SMs) is not."""
    ql, pre = REFERENCE_CASES[2]
    small = small_batch(ql, pre, seed=20260930)
    run_gpu(small, 4)
    assert _split_slots() > 0
    q, kv = lengths_chunked_4k()
    run_gpu(build_attention_batch(q, kv), 4)
    assert _split_slots() == 0


@pytest.mark.parametrize("splits", [4, 8, 16])
def test_uniform_splits_4k_against_oracle(monkeypatch, splits):
    """B200_ATTN_SPLIT_UNIFORM=1 splits every query unit of the 4K config
    `splits` ways (the reference's rule): the split path at full size, every
    sequence's sampled rows against the oracle."""
    monkeypatch.setenv("B200_ATTN_SPLIT_UNIFORM", "1")
    q, kv = lengths_chunked_4k()
    batch = build_attention_batch(q, kv)
    want, rows = sampled_oracle(batch, sample_blocks(q))
    got = run_gpu(batch, splits)
    assert _split_slots() == 64 * 16 * 2  # every (query unit, KV head) of the batch
    assert_close(got[rows], want, f"4k uniform S={splits}")
    _no_device_error()


def test_full_16k_config_every_sequence_against_oracle():
    """The 16K config at full size (64 sequences, 2048-token chunks, KV
    8192-16384): the first, middle and last 16 rows of every sequence against
    the oracle at S = 1, 4 and 8 and with every query unit split 4 ways, and
    the split runs against S = 1 over every row (a size-independent property)."""
    q, kv = lengths_chunked_16k()
    batch = build_attention_batch(q, kv)
    want, rows = sampled_oracle(batch, sample_blocks(q))
    outs = {s: run_gpu(batch, s) for s in (1, 4, 8)}
    with pytest.MonkeyPatch.context() as mp:  # every query unit split 4 ways
        mp.setenv("B200_ATTN_SPLIT_UNIFORM", "1")
        outs["4u"] = run_gpu(batch, 4)
    for s, got in outs.items():
        assert_close(got[rows], want, f"16k S={s}")
    for s in (4, 8, "4u"):
        mx, mn = errors(outs[s], outs[1])
        assert mx <= ATOL_MAX and mn <= 2e-4, (s, mx, mn)
    _no_device_error()


def test_mixed_256_every_shard_against_oracle():
    """The mixed batch (256 sequences, half decode rows, KV 512-16384) as the
    8-GPU run shards it (LPT by causal FLOPs): every shard built as its rank
    builds it and run on this GPU, sampled rows of every sequence and every
    decode row against the oracle; then the whole batch in one call."""
    from minicpm_b200.sharding import lpt_shard

    q, kv = lengths_mixed()
    shards = lpt_shard(q, kv, 8, 16, 128)
    assert sorted(i for ids in shards for i in ids) == list(range(len(q)))
    for rank, ids in enumerate(shards):
        batch = build_attention_batch([q[i] for i in ids], [kv[i] for i in ids], seq_ids=ids)
        want, rows = sampled_oracle(batch, sample_blocks(batch.query_lens))
        picked = set(rows.tolist())
        cu = batch.cu_seqlens_q.tolist()
        assert all(cu[j] in picked for j, n in enumerate(batch.query_lens) if n == 1)  # every decode row is checked
        for s in (0, 4):
            assert_close(run_gpu(batch, s)[rows], want, f"mixed shard {rank} S={s}")
    full = build_attention_batch(q, kv)
    want, rows = sampled_oracle(full, sample_blocks(q))
    assert_close(run_gpu(full, 0)[rows], want, "mixed whole batch")
    _no_device_error()


def test_split_combine_matches_reference_reduce(golden_dir):
    import numpy as np

    rec = np.load(golden_dir / "attn_small_b.npz")
    for s in rec["splits"].tolist():
        o = torch.from_numpy(rec[f"o_split_s{s}"]).cuda()
        m = torch.from_numpy(rec[f"m_split_s{s}"]).cuda()
        l = torch.from_numpy(rec[f"l_split_s{s}"]).cuda()
        want = torch.from_numpy(rec[f"reduce_s{s}"])
        out = torch.empty(o.shape[1:], device="cuda", dtype=torch.float32)
        split_kv_combine(o, m, l, out)
        assert (out.cpu() - want).abs().max().item() < 2e-6
        out16 = torch.empty(o.shape[1:], device="cuda", dtype=torch.bfloat16)
        split_kv_combine(o.to(torch.bfloat16), m, l, out16)
        assert (out16.cpu().float() - want).abs().max().item() < 2e-2


@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("num_splits", [1, 2, 3, 5, 8, 13, 16])
@pytest.mark.parametrize("partial_dtype", [torch.float32, torch.bfloat16])
def test_split_combine_shapes_against_oracle(head_dim, num_splits, partial_dtype):
    """The combine over every split bound (4 / 8 / 16) and row-group width
    (head_dim / 8 threads per row), with inactive splits holding NaN, rows
    with no active split, and a row count that leaves a partial block."""
    from oracle import split_kv_reduce_reference

    gen = torch.Generator().manual_seed(1000 * head_dim + num_splits)
    t, h = 37, 3  # 111 rows: not a multiple of any block's row count
    o = torch.randn(num_splits, t, h, head_dim, generator=gen)
    m = torch.randn(num_splits, t, h, generator=gen) * 4
    l = torch.rand(num_splits, t, h, generator=gen) * 50 + 0.5
    inactive = torch.rand(num_splits, t, h, generator=gen) < 0.3
    inactive[:, 5, 1] = True  # a row with no active split at all
    l[inactive] = 0.0
    m[inactive] = float("-inf")
    o[inactive] = float("nan")
    want = split_kv_reduce_reference(o, m, l)
    out_dtype = torch.float32 if partial_dtype == torch.float32 else torch.bfloat16
    out = torch.empty(t, h, head_dim, device="cuda", dtype=out_dtype)
    split_kv_combine(o.to(partial_dtype).cuda(), m.cuda(), l.cuda(), out)
    torch.cuda.synchronize()
    got = out.float().cpu()
    assert torch.isfinite(got).all()
    assert torch.equal(got[5, 1], torch.zeros(head_dim))
    tol = 2e-5 if partial_dtype == torch.float32 else 2e-2
    assert (got - want).abs().max().item() <= tol


@pytest.mark.parametrize("hq,hkv", [(16, 2), (8, 8), (16, 1), (12, 2), (32, 16)])
def test_head_dim_64_against_oracle(hq, hkv):
    """head_dim 64 (accepted by the reference wrapper): the kernel's narrow
    variant (K/V half-slots, K = 64 S UMMAs, N = 64 P V UMMAs), with per-KV-head
    maps and, at 16 KV heads, the 4-D maps; partial pages, a decode row,
    splits 1 / 4 / auto and every unit split 4 ways."""
    batch = small_batch([37, 1, 100, 16, 300], [200, 63, 1000, 0, 2500], seed=64, num_q_heads=hq, num_kv_heads=hkv,
                        head_dim=64)
    want = oracle(batch)
    for s in (1, 4, 0):
        assert_close(run_gpu(batch, s), want, f"d64 {hq}/{hkv} S={s}")
    with pytest.MonkeyPatch.context() as mp:
        mp.setenv("B200_ATTN_SPLIT_UNIFORM", "1")
        assert_close(run_gpu(batch, 4), want, f"d64 {hq}/{hkv} uniform S=4")
    _no_device_error()


def test_head_dim_64_chunked_prefill():
    """head_dim 64 on 8 sequences of the 4K config: sampled rows of every
    sequence against the oracle, and NaN in the page tails."""
    q, kv = lengths_chunked_4k(num_seqs=8)
    batch = build_attention_batch(q, kv, head_dim=64)
    want, rows = sampled_oracle(batch, sample_blocks(q))
    assert_close(run_gpu(batch, 0)[rows], want, "d64 4k")
    cache = batch.kv_cache.clone()
    for row, L in enumerate(batch.kv_lens):
        if L % 16:
            cache[int(batch.block_table[row, (L - 1) // 16]), :, L % 16:] = float("nan")
    batch.kv_cache = cache
    assert_close(run_gpu(batch, 0)[rows], want, "d64 4k nan tails")
    _no_device_error()


def test_head_dim_64_decode_batch_and_dispatcher(monkeypatch):
    """A head_dim-64 batch of decode rows takes the prefill kernel (the decode
    kernel is built for 128); through the dispatcher with the 5-D cache."""
    batch = small_batch([1, 1, 1], [5, 700, 2048], seed=65, head_dim=64)
    assert_close(run_gpu(batch, 0), oracle(batch), "d64 decode rows")
    b = small_batch([20, 33], [100, 400], seed=66, head_dim=64).to("cuda")
    out = torch.empty_like(b.q)
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    iluvatar_attention(b.q, b.kv_cache, b.kv_cache, out, b.cu_seqlens_q, b.max_seqlen_q, b.seqused_k, b.max_seqlen_k,
                       b.softmax_scale, causal=True, block_table=b.block_table)
    torch.cuda.synchronize()
    cpu = small_batch([20, 33], [100, 400], seed=66, head_dim=64)
    assert_close(out.cpu(), oracle(cpu), "d64 dispatcher")
    _no_device_error()


@pytest.mark.parametrize("hq,hkv", [(16, 2), (8, 8), (16, 1), (12, 2), (32, 16)])
def test_head_dim_256_against_oracle(hq, hkv):
    """head_dim 256 (accepted by the reference wrapper,
    kernels/triton_split_kv_paged.py:270): the kernel's wide variant, one
    query tile per unit, K and V in two 128-column halves; partial pages, a
    decode row, splits 1 / 4 / auto and every unit split 4 ways."""
    batch = small_batch([37, 1, 100, 16, 300], [200, 63, 1000, 0, 2500], seed=256, num_q_heads=hq, num_kv_heads=hkv,
                        head_dim=256)
    want = oracle(batch)
    for s in (1, 4, 0):
        assert_close(run_gpu(batch, s), want, f"d256 {hq}/{hkv} S={s}")
    with pytest.MonkeyPatch.context() as mp:
        mp.setenv("B200_ATTN_SPLIT_UNIFORM", "1")
        assert_close(run_gpu(batch, 4), want, f"d256 {hq}/{hkv} uniform S=4")
    _no_device_error()


def test_head_dim_256_chunked_prefill_and_dispatcher(monkeypatch):
    """head_dim 256 on 8 sequences of the 4K config (sampled rows of every
    sequence against the oracle), fp16, decode rows, and a call through the
    dispatcher with the 5-D cache."""
    q, kv = lengths_chunked_4k(num_seqs=8)
    batch = build_attention_batch(q, kv, head_dim=256)
    want, rows = sampled_oracle(batch, sample_blocks(q))
    assert_close(run_gpu(batch, 0)[rows], want, "d256 4k")
    half = small_batch([40, 3], [200, 77], seed=257, head_dim=256, dtype=torch.float16)
    assert_close(run_gpu(half, 1), oracle(half), "d256 fp16")
    dec = small_batch([1, 1, 1], [5, 700, 2048], seed=258, head_dim=256)
    assert_close(run_gpu(dec, 0), oracle(dec), "d256 decode rows")
    b = small_batch([20, 33], [100, 400], seed=259, head_dim=256).to("cuda")
    out = torch.empty_like(b.q)
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    iluvatar_attention(b.q, b.kv_cache, b.kv_cache, out, b.cu_seqlens_q, b.max_seqlen_q, b.seqused_k, b.max_seqlen_k,
                       b.softmax_scale, causal=True, block_table=b.block_table)
    torch.cuda.synchronize()
    assert_close(out.cpu(), oracle(small_batch([20, 33], [100, 400], seed=259, head_dim=256)), "d256 dispatcher")
    _no_device_error()


@pytest.mark.parametrize("head_dim", [64, 256])
def test_head_sizes_with_page_size_32_int64_and_a_wide_table(head_dim):
    """head_dim 64 and 256 with 32-token pages (two 16-key slices per page),
    int64 block table and lengths, and a block table wider than needed."""
    batch = small_batch([33, 7, 150], [100, 500, 1300], seed=head_dim + 5, block_size=32, extra_table_cols=5,
                        head_dim=head_dim)
    want = oracle(batch)
    b = batch.to("cuda")
    for s in (1, 4):
        out = torch.empty_like(b.q)
        paged_split_kv_attention(b.q, b.kv_cache[:, 0], b.kv_cache[:, 1], out, b.block_table.long(), b.seqused_k.long(),
                                 b.cu_seqlens_q.long(), b.max_seqlen_q, b.max_seqlen_k, b.softmax_scale, num_splits=s)
        torch.cuda.synchronize()
        assert_close(out.cpu(), want, f"d{head_dim} bs32 int64 S={s}")
    _no_device_error()
