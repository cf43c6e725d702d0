"""Sequence sharding of a paged prefill batch over one process per GPU.

Sequences are independent in causal paged attention, so a batch splits by
sequence with no exchange on the hot path: every rank builds its own page
pool, block table, ``cu_seqlens_q`` and ``seqused_k`` for its sequences and
runs the kernel on them.  A collective is used only to gather outputs for
verification (``gather_rows_to_rank0``), never inside a timed step.

* ``contiguous_shard`` -- equal contiguous counts (the fixed-shape chunked
  prefill batches).
* ``lpt_shard`` -- longest-processing-time assignment by the causal FLOP count
  of ``tests/attention_harness.py:381-385`` of the reference (the mixed batch
  with decode rows, whose per-sequence cost varies by orders of magnitude).
"""

from __future__ import annotations

import heapq
from typing import Sequence

import torch


def contiguous_shard(num_seqs: int, world: int, rank: int) -> list[int]:
    """Sequence ids of ``rank``: a contiguous block, sizes differing by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(num_seqs, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def sequence_cost(q_len: int, kv_len: int, num_q_heads: int, head_dim: int) -> int:
    prior = kv_len - q_len
    return 4 * (q_len * prior + q_len * (q_len + 1) // 2) * num_q_heads * head_dim


def lpt_shard(query_lens: Sequence[int], kv_lens: Sequence[int], world: int, num_q_heads: int = 16,
              head_dim: int = 128) -> list[list[int]]:
    """Assign sequences to ``world`` ranks, heaviest first onto the least-loaded rank.

    Deterministic (ties broken by sequence id, then rank id); each rank's ids are
    returned sorted.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    costs = [sequence_cost(q, k, num_q_heads, head_dim) for q, k in zip(query_lens, kv_lens)]
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(x) for x in out]


def shard_loads(query_lens, kv_lens, shards, num_q_heads: int = 16, head_dim: int = 128) -> list[int]:
    return [sum(sequence_cost(query_lens[i], kv_lens[i], num_q_heads, head_dim) for i in ids) for ids in shards]


def gather_rows_to_rank0(out: torch.Tensor, world: int, rank: int) -> torch.Tensor | None:
    """Concatenate every rank's ``[T_r, H, D]`` output on rank 0 (verification only).

    Uses ``all_gather`` of the row counts, then of zero-padded row blocks, on the
    default process group (NCCL for GPU tensors, gloo for CPU tensors).
    Returns the concatenation in rank order on rank 0, ``None`` elsewhere.
    """
    if world == 1:
        return out
    import torch.distributed as dist

    n = torch.tensor([out.shape[0]], device=out.device, dtype=torch.int64)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n)
    counts = [int(c.item()) for c in counts]
    cap = max(counts)
    padded = torch.zeros((cap,) + tuple(out.shape[1:]), device=out.device, dtype=out.dtype)
    padded[: out.shape[0]] = out
    blocks = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(blocks, padded)
    if rank != 0:
        return None
    return torch.cat([b[:c] for b, c in zip(blocks, counts)], dim=0)


__all__ = ["contiguous_shard", "lpt_shard", "sequence_cost", "shard_loads", "gather_rows_to_rank0"]
