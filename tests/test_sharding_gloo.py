"""Sequence sharding over ranks, tested with world_size-2 gloo process groups on CPU.

Each rank builds only its own sequences (own page pool, block table,
cu_seqlens_q, seqused_k), computes its rows (here with the CPU oracle, which
stands in for the kernel: what is under test is the host-side partition and
the verification gather), and the gathered result must equal the
single-process result over the whole batch row for row.  A rank that fails
before the gather makes the survivor's collective end with an error within
the process-group timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from minicpm_b200.sharding import contiguous_shard, lpt_shard, shard_loads
from minicpm_b200.workloads import build_attention_batch, lengths_mixed

ROOT = Path(__file__).resolve().parent.parent


def test_contiguous_shard_covers_everything_once():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            ids = [i for r in range(world) for i in contiguous_shard(n, world, r)]
            assert ids == list(range(n))
            sizes = [len(contiguous_shard(n, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_lpt_balances_the_mixed_batch():
    q, kv = lengths_mixed()
    shards = lpt_shard(q, kv, 8)
    assert sorted(i for s in shards for i in s) == list(range(len(q)))
    loads = shard_loads(q, kv, shards)
    assert max(loads) / (sum(loads) / 8) < 1.02  # within 2% of perfect balance
    assert lpt_shard(q, kv, 8) == shards  # deterministic


def test_per_sequence_content_is_shard_independent():
    q, kv = [5, 9, 3], [30, 40, 20]
    full = build_attention_batch(q, kv)
    part = build_attention_batch(q[1:], kv[1:], seq_ids=[1, 2])
    assert torch.equal(full.q[5:], part.q)
    for j, sid in enumerate((1, 2)):
        a = full.kv_cache[full.block_table[sid, : (kv[sid] + 15) // 16].long()]
        b = part.kv_cache[part.block_table[j, : (kv[sid] + 15) // 16].long()]
        assert torch.equal(a, b)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, result_q):
    try:
        sys.path[:0] = [str(ROOT), str(ROOT / "minicpm-attention-optimization-iluvatar_b200")]
        import datetime

        import torch.distributed as dist

        from minicpm_b200.sharding import gather_rows_to_rank0, lpt_shard
        from minicpm_b200.workloads import build_attention_batch
        from oracle import paged_attention_reference

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.set_num_threads(1)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        q = [40, 1, 17, 1, 90, 3]
        kv = [200, 300, 17, 1000, 120, 64]
        ids = lpt_shard(q, kv, world)[rank]
        batch = build_attention_batch([q[i] for i in ids], [kv[i] for i in ids], seq_ids=ids,
                                      num_q_heads=4, num_kv_heads=2, head_dim=64)
        out = paged_attention_reference(batch.q, batch.k_cache, batch.v_cache, batch.block_table,
                                        batch.cu_seqlens_q, batch.seqused_k, batch.softmax_scale)
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # leaves before the gather
        ids_t = torch.tensor(ids, dtype=torch.int64)
        gathered = gather_rows_to_rank0(out, world, rank)
        all_ids = [torch.zeros(6, dtype=torch.int64) for _ in range(world)]
        padded = torch.full((6,), -1, dtype=torch.int64)
        padded[: len(ids)] = ids_t
        dist.all_gather(all_ids, padded)
        # The bench's cross-rank reductions of a per-rank time (a collective
        # each, in the same order on every rank).
        import bench

        x = 10.0 + 5.0 * rank
        red = (bench.max_over_ranks(x, world), bench.sum_over_ranks(x, world), bench.gather_over_ranks(x, world))
        if rank == 0:
            order = [int(i) for t in all_ids for i in t.tolist() if i >= 0]
            result_q.put(("ok", order, gathered.numpy().copy(), red))
        dist.destroy_process_group()
    except SystemExit:
        raise
    except Exception as exc:  # reported to the parent
        result_q.put(("error", rank, f"{type(exc).__name__}: {exc}", traceback.format_exc()))


def _spawn(mode):
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    # Drain the queue before joining: a child cannot exit while its queued
    # data is still waiting in the pipe.
    import queue as _queue
    import time as _time

    results = []
    deadline = _time.time() + 120
    while _time.time() < deadline and (any(p.is_alive() for p in procs) or not result_q.empty()):
        try:
            results.append(result_q.get(timeout=0.5))
        except _queue.Empty:
            pass
    for p in procs:
        p.join(timeout=10)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return procs, results


@pytest.mark.timeout(300)
def test_gloo_two_ranks_gather_matches_single_process():
    procs, results = _spawn("ok")
    assert all(p.exitcode == 0 for p in procs), [r for r in results if r[0] == "error"]
    (_, order, gathered, red), = [r for r in results if r[0] == "ok"]
    assert red == (15.0, 25.0, [10.0, 15.0])
    import bench

    spread = bench.rank_spread(red[2], 5)
    assert spread["min_ms"] == 2.0 and spread["max_ms"] == 3.0 and spread["max_over_min"] == 1.5
    from oracle import paged_attention_reference

    q = [40, 1, 17, 1, 90, 3]
    kv = [200, 300, 17, 1000, 120, 64]
    batch = build_attention_batch([q[i] for i in order], [kv[i] for i in order], seq_ids=order,
                                  num_q_heads=4, num_kv_heads=2, head_dim=64)
    want = paged_attention_reference(batch.q, batch.k_cache, batch.v_cache, batch.block_table, batch.cu_seqlens_q,
                                     batch.seqused_k, batch.softmax_scale)
    assert torch.equal(torch.from_numpy(gathered), want)


@pytest.mark.timeout(300)
def test_gloo_rank_failure_surfaces_as_error_not_hang():
    procs, results = _spawn("fail")
    assert procs[1].exitcode == 3
    errors = [r for r in results if r[0] == "error"]
    assert errors and errors[0][1] == 0, results  # rank 0's collective failed with an error
