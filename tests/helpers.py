"""Shared helpers for the parity tests: run the CUDA path and the oracle on one batch."""

from __future__ import annotations

import math

import torch

from minicpm_b200 import paged_split_kv_attention
from minicpm_b200.workloads import AttentionBatch, build_attention_batch
from oracle import paged_attention_reference

# Tolerances: bf16 attention output against the fp32 oracle.  Max-abs 2e-2
# is the target's bound (tighter than the reference test's 0.05); mean-abs
# 1e-3 is the reference test's own gate (tests/test_paged_split_kv.py:95).
ATOL_MAX = 2e-2
ATOL_MEAN = 1e-3


def run_gpu(batch: AttentionBatch, num_splits: int, device="cuda", dtype=None) -> torch.Tensor:
    b = batch.to(device)
    q = b.q if dtype is None else b.q.to(dtype)
    cache = b.kv_cache if dtype is None else b.kv_cache.to(dtype)
    out = torch.empty_like(q)
    paged_split_kv_attention(
        q, cache[:, 0], cache[:, 1], out, b.block_table, b.seqused_k, b.cu_seqlens_q,
        b.max_seqlen_q, b.max_seqlen_k, b.softmax_scale, num_splits=num_splits,
    )
    torch.cuda.synchronize()
    return out.cpu()


def oracle(batch: AttentionBatch) -> torch.Tensor:
    return paged_attention_reference(
        batch.q, batch.k_cache, batch.v_cache, batch.block_table, batch.cu_seqlens_q, batch.seqused_k, batch.softmax_scale
    )


def errors(got: torch.Tensor, want: torch.Tensor) -> tuple[float, float]:
    d = (got.float() - want.float()).abs()
    return d.max().item(), d.mean().item()


def assert_close(got: torch.Tensor, want: torch.Tensor, tag: str = "", atol_max=ATOL_MAX, atol_mean=ATOL_MEAN):
    assert torch.isfinite(got.float()).all(), f"{tag}: non-finite output"
    mx, mn = errors(got, want)
    assert mx <= atol_max and mn <= atol_mean, f"{tag}: max_error={mx:.5f} mean_error={mn:.6f}"
    return mx, mn


def row_subset_batch(batch: AttentionBatch, seq: int, r0: int, r1: int) -> tuple[AttentionBatch, slice]:
    """Query rows [r0, r1) of one sequence as a batch of its own for the oracle.

    The rows keep their absolute positions: the sub-batch's KV length is the
    causal limit of row r1 - 1.
    """
    q_len = batch.query_lens[seq]
    L = batch.kv_lens[seq]
    begin = int(batch.cu_seqlens_q[seq])
    sub_len = L - q_len + r1
    sub = AttentionBatch(
        q=batch.q[begin + r0 : begin + r1],
        kv_cache=batch.kv_cache,
        block_table=batch.block_table[seq : seq + 1],
        cu_seqlens_q=torch.tensor([0, r1 - r0], dtype=torch.int32),
        seqused_k=torch.tensor([sub_len], dtype=torch.int32),
        query_lens=[r1 - r0],
        kv_lens=[sub_len],
        softmax_scale=batch.softmax_scale,
        seq_ids=[batch.seq_ids[seq]],
    )
    return sub, slice(begin + r0, begin + r1)


def sample_blocks(query_lens, block: int = 16) -> list[tuple[int, int, int]]:
    """``(seq, r0, r1)`` row blocks: the first, middle and last ``block`` query
    rows of every sequence (every row of a sequence shorter than 3 blocks)."""
    picks = []
    for seq, q_len in enumerate(query_lens):
        if q_len <= 0:
            continue
        if q_len <= 3 * block:
            picks.append((seq, 0, q_len))
            continue
        mid = (q_len - block) // 2
        picks += [(seq, 0, block), (seq, mid, mid + block), (seq, q_len - block, q_len)]
    return picks


def sampled_oracle(batch: AttentionBatch, picks) -> tuple[torch.Tensor, torch.Tensor]:
    """The oracle on the picked row blocks only, in one call.

    Each block becomes a sequence of its own that keeps its rows' absolute
    positions (KV length = the causal limit of its last row, same block-table
    row).  Returns ``(want [N, H, D] fp32, row indices [N] into batch.q)``.
    """
    cu = batch.cu_seqlens_q.tolist()
    qs, rows, tables, lens, qlens = [], [], [], [], []
    for seq, r0, r1 in picks:
        begin = cu[seq]
        qs.append(batch.q[begin + r0 : begin + r1])
        rows.append(torch.arange(begin + r0, begin + r1))
        tables.append(batch.block_table[seq])
        lens.append(batch.kv_lens[seq] - batch.query_lens[seq] + r1)
        qlens.append(r1 - r0)
    sub = AttentionBatch(
        q=torch.cat(qs), kv_cache=batch.kv_cache, block_table=torch.stack(tables),
        cu_seqlens_q=torch.tensor([0, *torch.tensor(qlens).cumsum(0).tolist()], dtype=torch.int32),
        seqused_k=torch.tensor(lens, dtype=torch.int32), query_lens=qlens, kv_lens=lens,
        softmax_scale=batch.softmax_scale, seq_ids=[batch.seq_ids[p[0]] for p in picks],
    )
    return oracle(sub), torch.cat(rows)


def small_batch(query_lens, prefix_lens, **kw) -> AttentionBatch:
    return build_attention_batch(query_lens, [p + q for p, q in zip(prefix_lens, query_lens)], **kw)


__all__ = [
    "ATOL_MAX",
    "ATOL_MEAN",
    "run_gpu",
    "oracle",
    "errors",
    "assert_close",
    "row_subset_batch",
    "sample_blocks",
    "sampled_oracle",
    "small_batch",
    "math",
]
