"""Benchmark of the sm_100a paged prefill attention (and the RoPE + KV-cache write).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--splits S]
    python bench.py --impl reference ...   # the CPU implementation of the path, timed on host cores

Default workload: chunked prefill at 16K context -- 64 sequences, 2048-token
query chunks, total KV length uniform in [8192, 16384], 16 query heads / 2 KV
heads, head_dim 128, bf16, page size 16, permuted block table.  Under
torchrun the sequences are sharded over the ranks by causal FLOPs
(longest-processing-time first; one process per GPU, no collective in the
timed region); the reported value is the causal FLOPs of all ranks divided by
the slowest rank's device time.  The line's ``sub`` object carries the rest of
the metric from the same run: the 4K config at S = auto / 4 / 8, the mixed
256-sequence batch, the RoPE + KV-cache write at rotary_dim 64 / 128 x NeoX /
interleaved and the Split-KV combine, each with its roofline fraction.

One JSON line on rank 0.  ``value``: device-resident throughput (inputs in HBM
before the timed region).  ``e2e``: the same metric through the public
operator API (``iluvatar_attention``) with the inputs copied from pinned host
memory and the output copied back inside the timed region; the sequences go
in groups whose host-to-device copies, attention calls and read-backs overlap
on three streams.  Other workloads: the 4K batch, the mixed batch, the decode
batches, the RoPE + KV-cache write, the service's cache write and the Split-KV
combine alone (``--workload``).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "minicpm-attention-optimization-iluvatar_b200"
for _p in (str(ROOT), str(PKG_DIR)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "paged prefill attention TFLOP/s & tokens/s at 4K/16K ctx, 64 seqs, 1/2/4/8 B200; % TC peak"
HEAD_DIM = 128  # attention workloads; --head-dim 64 / 256 measures the other head sizes on the same shapes
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="chunked_prefill_16k",
                    choices=["chunked_prefill_16k", "chunked_prefill_4k", "mixed_256", "decode_16k", "decode_4k",
                             "rope_16384", "kv_write_16384", "split_combine_4k"])
    ap.add_argument("--splits", type=int, default=0, help="0 = automatic")
    ap.add_argument("--head-dim", type=int, default=128, choices=[64, 128, 256],
                    help="attention workloads: head size (the headline is 128)")
    ap.add_argument("--kv-quant", default="none", choices=["none", "fp8"],
                    help="attention workloads: an fp8 per-tensor KV cache (pages dequantised, then the kernel)")
    ap.add_argument("--num-seqs", type=int, default=0,
                    help="keep only the first N sequences of the workload (small cases for profiling)")
    ap.add_argument("--rotary-dim", type=int, default=128)
    ap.add_argument("--interleaved", action="store_true")
    ap.add_argument("--kv-dtype", default="auto",
                    choices=["auto", "fp8", "int8_per_token_head", "fp8_per_token_head"],
                    help="kv_write_16384: the cache kind; rope_16384 --service: auto or fp8")
    ap.add_argument("--service", action="store_true",
                    help="rope_16384: the service's rope-and-cache call (key rotated in place)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--graph", action="store_true",
                    help="attention workloads: time the K calls as one CUDA graph replay (no host launch gaps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="16K workload: skip the 4K / mixed / RoPE / combine entries of the line's \"sub\" object")
    ap.add_argument("--verify", action="store_true",
                    help="gather outputs to rank 0 (NCCL) and compare with one single-GPU call (default with >1 GPU)")
    ap.add_argument("--no-verify", action="store_true", help="skip that comparison with more than one GPU")
    return ap.parse_args()


# --------------------------------------------------------------------- ranks
def pin_to_gpu_numa_node(local: int) -> None:
    """Run this rank on the host cores next to its GPU (the PCI device's
    ``local_cpulist``), so the pinned host buffers of the e2e copies are
    first-touched on that NUMA node; a no-op where sysfs does not say."""
    try:
        prop = torch.cuda.get_device_properties(local)
        bdf = f"{prop.pci_domain_id:04x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
        text = Path(f"/sys/bus/pci/devices/{bdf}/local_cpulist").read_text().strip()
        cpus = set()
        for part in text.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
    except Exception:
        pass


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        pin_to_gpu_numa_node(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def _reduce_device():
    """Where the small reductions run: the GPU under NCCL, the host under gloo."""
    import torch.distributed as dist

    return "cuda" if dist.get_backend() == "nccl" else "cpu"


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device=_reduce_device(), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(x: float, world: int) -> list:
    """Every rank's value of x, in rank order (a collective: all ranks call it)."""
    if world == 1:
        return [x]
    import torch.distributed as dist

    t = torch.tensor([x], device=_reduce_device(), dtype=torch.float64)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [float(p.item()) for p in parts]


def rank_spread(rank_ms: list, steps: int) -> dict:
    """Per-rank device time per call: the load balance of the sharding."""
    per = [m / steps for m in rank_ms]
    return {"min_ms": min(per), "max_ms": max(per), "max_over_min": max(per) / min(per),
            "per_rank_ms": [round(x, 4) for x in per]}


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device=_reduce_device(), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------------- peaks / clocks
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        rows = []
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]) if parts[3] not in ("[N/A]", "") else None,
                                 active=parts[4], hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        if not rows:
            return None
        loaded = [r for r in rows if r["power"] is None or r["power"] > 200] or rows
        reasons = set()
        for r in loaded:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                              ("pcap", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(loaded)}


# --------------------------------------------------------------------- workloads
def build_local_batch(workload: str, world: int, rank: int, num_seqs: int = 0):
    """This rank's sequences: longest-processing-time assignment by causal FLOPs
    (the KV lengths of one batch vary 2x to 30x, so equal counts leave the
    slowest rank well behind the mean)."""
    from minicpm_b200 import workloads
    from minicpm_b200.sharding import lpt_shard

    q, kv = workloads.WORKLOADS[workload]()
    if num_seqs:
        q, kv = q[:num_seqs], kv[:num_seqs]
    ids = lpt_shard(q, kv, world, 16, HEAD_DIM)[rank]
    batch = workloads.build_attention_batch([q[i] for i in ids], [kv[i] for i in ids], seq_ids=ids, head_dim=HEAD_DIM)
    return batch, q, kv


def cpu_sample_flops(batch, rows: int):
    """Oracle over the last ``rows`` query rows of the batch's first sequence."""
    sys.path.insert(0, str(ROOT))
    from oracle import causal_flops, paged_attention_reference

    from minicpm_b200.workloads import AttentionBatch

    q_len, L = batch.query_lens[0], batch.kv_lens[0]
    r1, r0 = q_len, max(0, q_len - rows)
    sub = AttentionBatch(q=batch.q[r0:r1], kv_cache=batch.kv_cache, block_table=batch.block_table[:1],
                         cu_seqlens_q=torch.tensor([0, r1 - r0], dtype=torch.int32),
                         seqused_k=torch.tensor([L], dtype=torch.int32), query_lens=[r1 - r0], kv_lens=[L],
                         softmax_scale=batch.softmax_scale, seq_ids=batch.seq_ids[:1])
    flops = causal_flops([r1 - r0], [L], 16, HEAD_DIM)

    def run():
        paged_attention_reference(sub.q, sub.k_cache, sub.v_cache, sub.block_table, sub.cu_seqlens_q, sub.seqused_k,
                                  sub.softmax_scale, q_chunk=256)

    desc = f"oracle fp32 over query rows [{r0},{r1}) of sequence {batch.seq_ids[0]} (KV length {L})"
    return run, flops, desc


def time_cpu(run, reps: int):
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    return times


# --------------------------------------------------------------------- shared config
def attention_config(workload: str, world: int, splits: int, num_seqs: int = 0) -> dict:
    """The workload's ``config`` object, identical in both arms: the shapes and
    FLOPs of the whole job (all ranks), the split count the call resolves
    (``splits`` 0 = automatic), the sharding and the L2 note."""
    from minicpm_b200 import workloads
    from minicpm_b200.split_kv_paged import choose_num_splits
    from oracle import causal_flops  # FLOP formula of the reference harness (no compute)

    q, kv = workloads.WORKLOADS[workload]()
    if num_seqs:
        q, kv = q[:num_seqs], kv[:num_seqs]
    if splits:
        resolved = splits
    else:
        from minicpm_b200.sharding import lpt_shard

        # rank 0's shard decides the automatic count the call resolves to
        ids = lpt_shard(q, kv, world, 16, HEAD_DIM)[0]
        resolved = choose_num_splits(sum(q[i] for i in ids), len(ids), 16, 2, max(kv[i] for i in ids))
    kv_mb = sum(workloads.attention_kv_bytes([0], [L], head_dim=HEAD_DIM) for L in kv) / 1e6 / world
    q_mb = sum(q) * 16 * HEAD_DIM * 2 / 1e6 / world
    return {
        "workload": workload,
        "seqs": len(q),
        "query_tokens": sum(q),
        "causal_flops": float(causal_flops(q, kv, 16, HEAD_DIM)),
        "heads": "16q/2kv", "head_dim": HEAD_DIM, "page_size": 16,
        "num_splits": resolved,
        "parallelism": f"sequence-sharded x{world} (LPT by causal FLOPs)",
        "l2": "inputs larger than L2 (KV %.0f MB + Q %.0f MB per GPU)" % (kv_mb, q_mb),
    }


# --------------------------------------------------------------------- reference arm
def reference_arm(args, world, rank):
    """The CPU implementation of the path (the fp32 oracle port), timed on host cores.

    Each step runs the oracle over a bounded sample of the workload (the last
    512 query rows of its first sequence, full causal KV context) and the rate
    is reported in the workload's own unit; ``config`` is the same object the
    sm_100a arm prints.
    """
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    if args.workload not in ("chunked_prefill_16k", "chunked_prefill_4k", "mixed_256"):
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm covers the prefill attention workloads"}))
        return
    from minicpm_b200 import workloads

    q, kv = workloads.WORKLOADS[args.workload]()
    batch = workloads.build_attention_batch(q[:1], kv[:1], seq_ids=[0], head_dim=HEAD_DIM)
    run, flops, desc = cpu_sample_flops(batch, 512)
    for _ in range(args.warmup):
        run()
    times = time_cpu(run, args.steps)
    total = sum(times)
    value = flops * args.steps / total / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) q/k/v, random-permuted page table)",
        "config": attention_config(args.workload, world, args.splits, args.num_seqs),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- RoPE bench
def rope_run(rotary_dim: int, is_neox: bool, service: bool, kv_dtype: str, steps: int, warmup: int, local: int,
             world: int, clocks: bool = True) -> dict:
    """Graph-timed RoPE + paged KV-cache write of 16384 tokens on this GPU.

    The reference operator, or with ``service`` the service's call (key rotated
    in place; ``kv_dtype`` "fp8" caches).  Returns GB/s of this GPU, the device
    time per launch, the algorithmic bytes and the clock record.
    """
    from minicpm_b200 import fused_rope_and_cache, kv_cache
    from minicpm_b200.workloads import build_rope_batch, rope_algorithmic_bytes

    dev = torch.device("cuda", local)
    b = build_rope_batch(16384, rotary_dim=rotary_dim, is_neox=is_neox)
    g = b.to(dev)
    nbytes = rope_algorithmic_bytes(b)
    fp8 = service and kv_dtype == "fp8"
    if service:
        t, hkv, d = b.key.shape
        written = int((b.slot_mapping >= 0).sum())
        nbytes += 2 * t * hkv * rotary_dim * b.key.element_size()  # rotated key written back
        if fp8:
            nbytes -= 2 * written * hkv * d * (b.key.element_size() - 1)  # 1-byte cache rows
            g.key_cache = torch.zeros(g.key_cache.shape, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
            g.value_cache = torch.zeros_like(g.key_cache)
        ks = torch.tensor([0.02], device=dev)
        vs = torch.tensor([0.015], device=dev)

    def step(i):
        if service:
            kv_cache.rope_and_cache(g.query, g.key, g.value, g.positions, g.cos_sin_cache, g.is_neox, g.key_cache,
                                    g.value_cache, g.slot_mapping, ks, vs, True, fp8)
        else:
            fused_rope_and_cache(g.query, g.key, g.value, g.positions, g.cos_sin_cache, g.is_neox, g.key_cache,
                                 g.value_cache, g.slot_mapping)

    for i in range(warmup):
        step(i)
    # Back-to-back launches replayed from a CUDA graph: the ~170 MB one launch
    # moves exceed the 126 MB L2, so each launch streams from HBM.
    ms, clk = graph_timed(step, steps, local, world, clocks=clocks)
    return {"gbs": nbytes / (ms * 1e-3) / 1e9, "ms": ms, "nbytes": nbytes, "clocks": clk, "batch": b, "fp8": fp8}


def rope_bench(args, world, rank, local):
    """RoPE + paged KV-cache write of 16384 tokens (the reference operator, or with
    ``--service`` the service's call: key rotated in place, ``--kv-dtype fp8`` caches)."""
    r = rope_run(args.rotary_dim, not args.interleaved, args.service, args.kv_dtype, args.steps, args.warmup, local,
                 world)
    peaks, kind = measured_peaks()
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = rope_cpu_baseline(r["batch"], r["nbytes"])
    if rank == 0:
        line = {
            "metric": "RoPE + paged KV-cache write GB/s", "value": r["gbs"] * world, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "rope_16384", "tokens": 16384, "rotary_dim": args.rotary_dim,
                       "is_neox": not args.interleaved, "service": bool(args.service),
                       "cache": "fp8_e4m3" if r["fp8"] else "bf16", "algorithmic_bytes": r["nbytes"],
                       "l2": "inputs larger than L2, back-to-back launches",
                       "timing": "CUDA graph of all timed launches, replayed once"},
            "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": r["gbs"] / peaks["hbm_gbs"], "traffic": None, "peak_kind": kind},
            "clocks": r["clocks"],
            "gpu_launches": args.steps,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def rope_cpu_baseline(b, nbytes):
    """The oracle's RoPE + cache write on the first 2048 of the 16384 tokens, on the host cores."""
    from oracle import rope_and_cache_reference

    torch.set_num_threads(os.cpu_count() or 1)
    n = 2048

    def run():
        rope_and_cache_reference(b.query[:n], b.key[:n], b.value[:n], b.positions[:n], b.cos_sin_cache, b.is_neox,
                                 b.key_cache, b.value_cache, b.slot_mapping[:n], b.rotary_dim)

    run()
    times = time_cpu(run, 3)
    sec = sum(times) / len(times)
    return {"value": nbytes * n / b.query.shape[0] / sec / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"first {n} of 16384 tokens, 3 repetitions (bytes scaled to the sample)"}


# --------------------------------------------------------------------- graph-timed short kernels
def graph_timed(step, steps: int, local: int, world: int, clocks: bool = True):
    """Device time per launch of ``step(i)``, i = 0..steps-1, captured in one CUDA graph.

    Kernels of a few to tens of microseconds launched one by one from Python
    would be timed behind the host's launch overhead; replaying the captured
    sequence keeps the GPU busy back to back.  Returns (ms per launch, clocks).
    """
    stream = torch.cuda.Stream(device=local)
    stream.wait_stream(torch.cuda.current_stream(local))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                step(i)
    torch.cuda.current_stream(local).wait_stream(stream)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(local)
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if clocks else None
    if sampler:
        sampler.__enter__()
    try:
        s.record()
        graph.replay()
        e.record()
        e.synchronize()
    finally:
        if sampler:
            sampler.__exit__(None, None, None)
    ms = max_over_ranks(s.elapsed_time(e) / steps, world)
    del graph
    return ms, (sampler.summary() if sampler else None)


# --------------------------------------------------------------------- KV-cache write bench
KV_ROTATION = 8  # distinct input sets cycled by the timed loop


def kv_write_bench(args, world, rank, local):
    """The service's cache update on 16384 new tokens (16 KV-head-dim rows of 2 heads each).

    One launch of 16384 tokens moves ~33 MB, less than the 126 MB L2, so the
    timed loop cycles through 8 independent batches (distinct K/V rows and slot
    sets; ~190 MB of distinct bytes with the 64 MB cache) back to back.
    """
    from minicpm_b200 import kv_cache
    from minicpm_b200.workloads import build_kv_write_batch, kv_write_algorithmic_bytes

    dev = torch.device("cuda", local)
    kind = args.kv_dtype
    first = build_kv_write_batch(16384, kv_cache_dtype=kind)
    shared_cache = first.kv_cache.to(dev)
    batches = []
    for r in range(KV_ROTATION):
        b = build_kv_write_batch(16384, kv_cache_dtype=kind, seed=1000 + r, num_blocks=4096)
        g = b.to(dev)
        g.kv_cache = shared_cache
        batches.append(g)
    nbytes = kv_write_algorithmic_bytes(first)

    def step(i):
        g = batches[i % KV_ROTATION]
        kc, vc = g.caches()
        if kind.endswith("per_token_head"):
            ks, vs = g.scale_cache_views()
            kv_cache.reshape_and_cache_flash_per_token_head_quant(g.key, g.value, kc, vc, ks, vs, g.slot_mapping)
        else:
            kv_cache.reshape_and_cache_flash(g.key, g.value, kc, vc, g.slot_mapping, kind, g.k_scale, g.v_scale)

    for i in range(max(args.warmup, KV_ROTATION)):
        step(i)
    # One step = one pass over the rotating input sets (KV_ROTATION launches).
    ms, clocks = graph_timed(step, args.steps * KV_ROTATION, local, world)
    peaks, pkind = measured_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = kv_write_cpu_baseline(first, nbytes)
    if rank == 0:
        line = {
            "metric": "paged KV-cache write GB/s", "value": gbs * world, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms * KV_ROTATION, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": str(first.key.dtype).replace("torch.", ""),
            "data": "synthetic",
            "config": {"workload": "kv_write_16384", "tokens": 16384, "kv_heads": 2, "head_dim": 128,
                       "kv_cache_dtype": kind, "algorithmic_bytes_per_launch": nbytes,
                       "launches_per_step": KV_ROTATION, "us_per_launch": ms * 1e3,
                       "timing": "CUDA graph of all timed launches, replayed once",
                       "l2": f"{KV_ROTATION} rotating input sets, footprint larger than L2, back-to-back launches"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "traffic": None, "peak_kind": pkind},
            "clocks": clocks,
            "gpu_launches": args.steps * KV_ROTATION,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def kv_write_cpu_baseline(b, nbytes):
    """The oracle's cache write of the same 16384 tokens, timed on the host cores."""
    from oracle import kv_write_reference

    torch.set_num_threads(os.cpu_count() or 1)
    kc, vc = b.caches()
    ksc = vsc = None
    if b.kv_cache_dtype.endswith("per_token_head"):
        ksc, vsc = (t.clone() for t in b.scale_cache_views())

    def run():
        kv_write_reference(b.key, b.value, kc, vc, b.slot_mapping, b.kv_cache_dtype, float(b.k_scale),
                           float(b.v_scale), ksc, vsc)

    run()
    times = time_cpu(run, 3)
    sec = sum(times) / len(times)
    return {"value": nbytes / sec / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": "the full 16384-token write, 3 repetitions"}


# --------------------------------------------------------------------- split-combine bench
def combine_run(s_count: int, steps: int, warmup: int, local: int, world: int, clocks: bool = True) -> dict:
    """Graph-timed cross-split reduce on the partials of the 4K chunked-prefill batch.

    32768 query tokens x 16 heads x 128, ``s_count`` partials in bf16 with fp32
    m/l, every split holding keys (l > 0), so every partial is read:
    algorithmic bytes = S*T*H*(D*2 + 8) read + T*H*D*2 written (688 MB at
    S = 4, larger than L2).
    """
    from minicpm_b200 import split_kv_combine

    dev = torch.device("cuda", local)
    t, h, d = 32768, 16, 128
    gen = torch.Generator().manual_seed(20260928)
    o = torch.randn(s_count, t, h, d, generator=gen).to(torch.bfloat16).to(dev)
    m = (torch.randn(s_count, t, h, generator=gen) * 3).to(dev)
    l = (torch.rand(s_count, t, h, generator=gen) * 100 + 1).to(dev)
    out = torch.empty(t, h, d, dtype=torch.bfloat16, device=dev)
    nbytes = s_count * t * h * (d * 2 + 8) + t * h * d * 2

    def step(i):
        split_kv_combine(o, m, l, out)

    for _ in range(warmup):
        step(0)
    ms, clk = graph_timed(step, steps, local, world, clocks=clocks)
    return {"gbs": nbytes / (ms * 1e-3) / 1e9, "ms": ms, "nbytes": nbytes, "clocks": clk, "o": o, "m": m, "l": l,
            "out": out, "shape": (t, h, d)}


def combine_bench(args, world, rank, local):
    """The Split-KV combine alone (``--splits`` partials, default 4) on 4K-batch-sized partials."""
    s_count = args.splits if args.splits > 1 else 4
    r = combine_run(s_count, args.steps, args.warmup, local, world)
    peaks, pkind = measured_peaks()
    t, h, d = r["shape"]
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        from oracle import split_kv_reduce_reference

        torch.set_num_threads(os.cpu_count() or 1)
        n = 2048
        oc, mc, lc = r["o"][:, :n].float().cpu(), r["m"][:, :n].cpu(), r["l"][:, :n].cpu()
        want = split_kv_reduce_reference(oc, mc, lc)
        got = r["out"][:n].float().cpu()
        assert (got - want).abs().max().item() <= 2e-2, "combine differs from the oracle"
        times = time_cpu(lambda: split_kv_reduce_reference(oc, mc, lc), 3)
        cpu = {"value": r["nbytes"] * n / t / (sum(times) / len(times)) / 1e9, "unit": "GB/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"first {n} of {t} tokens, 3 repetitions (bytes scaled to the sample)"}
    if rank == 0:
        line = {
            "metric": "Split-KV combine GB/s", "value": r["gbs"] * world, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "split_combine_4k", "tokens": t, "heads": h, "head_dim": d, "splits": s_count,
                       "algorithmic_bytes": r["nbytes"], "l2": "inputs larger than L2, back-to-back launches",
                       "timing": "CUDA graph of all timed launches, replayed once"},
            "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": r["gbs"] / peaks["hbm_gbs"], "traffic": None, "peak_kind": pkind},
            "clocks": r["clocks"],
            "gpu_launches": args.steps,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- verification
def verify_sharded(workload, num_seqs, batch, out, world, rank, splits):
    """Gather every rank's rows on rank 0 (NCCL) and compare them with one
    single-GPU call over the whole batch: a sequence's output does not depend
    on which rank or which physical pages hold it, so they must match bit for
    bit.  Returns the result on rank 0 (None elsewhere); raises on a mismatch."""
    import torch.distributed as dist

    from minicpm_b200 import paged_split_kv_attention, workloads
    from minicpm_b200.sharding import gather_rows_to_rank0

    full = gather_rows_to_rank0(out, world, rank)
    ids = [None] * world
    if world > 1:
        dist.all_gather_object(ids, list(batch.seq_ids))
    else:
        ids = [list(batch.seq_ids)]
    if rank != 0:
        return None
    order = [i for part in ids for i in part]
    q, kv = workloads.WORKLOADS[workload]()
    if num_seqs:
        q, kv = q[:num_seqs], kv[:num_seqs]
    ref = workloads.build_attention_batch([q[i] for i in order], [kv[i] for i in order], seq_ids=order,
                                          head_dim=HEAD_DIM).to(full.device)
    want = torch.empty_like(ref.q)
    paged_split_kv_attention(ref.q, ref.kv_cache[:, 0], ref.kv_cache[:, 1], want, ref.block_table, ref.seqused_k,
                             ref.cu_seqlens_q, ref.max_seqlen_q, ref.max_seqlen_k, ref.softmax_scale, num_splits=splits)
    torch.cuda.synchronize()
    same = bool(torch.equal(full, want))
    if not same:
        raise SystemExit("sharded output differs from the single-GPU output")
    return {"rows": int(full.shape[0]), "bit_identical_to_one_gpu": same, "gather": "NCCL all_gather to rank 0"}


# --------------------------------------------------------------------- e2e (host buffers)
E2E_MAX_GROUPS = 8
E2E_MIN_SEQS_PER_GROUP = 4   # with more than 16 sequences on the rank
E2E_MIN_GROUPS = 4           # fewer sequences: groups of one or two, so several groups are in flight


def split_into_groups(batch, n_groups: int):
    """Contiguous groups of the batch's sequences, each a batch of its own.

    Every group gets its own page pool holding exactly its sequences' pages,
    placed by a seeded permutation inside the pool (the block table stays a
    scattered physical mapping); Q rows, K/V values and lengths are the
    batch's own, so each group's output rows equal the batch's.
    """
    from minicpm_b200.workloads import AttentionBatch

    nseq = len(batch.query_lens)
    bounds = [round(i * nseq / n_groups) for i in range(n_groups + 1)]
    cu = batch.cu_seqlens_q.tolist()
    bs = batch.kv_cache.shape[2]
    parts = []
    for gi in range(n_groups):
        r0, r1 = bounds[gi], bounds[gi + 1]
        if r0 == r1:
            continue
        pages = [math.ceil(L / bs) for L in batch.kv_lens[r0:r1]]
        src = [batch.block_table[r, :n].long() for r, n in zip(range(r0, r1), pages)]
        src = torch.cat(src) if sum(pages) else torch.empty(0, dtype=torch.long)
        n = int(src.numel())
        slot = torch.randperm(max(n, 1), generator=torch.Generator().manual_seed(7919 + gi))[:n]
        pool = torch.zeros((max(n, 1),) + tuple(batch.kv_cache.shape[1:]), dtype=batch.kv_cache.dtype)
        pool[slot] = batch.kv_cache[src]
        table = torch.zeros(r1 - r0, max(max(pages), 1), dtype=torch.int32)
        off = 0
        for i, np_ in enumerate(pages):
            table[i, :np_] = slot[off:off + np_].to(torch.int32)
            off += np_
        parts.append(AttentionBatch(
            q=batch.q[cu[r0]:cu[r1]].contiguous(), kv_cache=pool, block_table=table,
            cu_seqlens_q=torch.tensor([c - cu[r0] for c in cu[r0:r1 + 1]], dtype=torch.int32),
            seqused_k=batch.seqused_k[r0:r1].clone(), query_lens=list(batch.query_lens[r0:r1]),
            kv_lens=list(batch.kv_lens[r0:r1]), softmax_scale=batch.softmax_scale,
            seq_ids=list(batch.seq_ids[r0:r1])))
    return parts


def e2e_pipelined(args, batch, out, splits, stream, world, total_flops, total_tokens):
    """The metric through ``iluvatar_attention`` with host-resident inputs and output.

    Each step copies every input from pinned host memory and reads ``out``
    back, inside the timed region.  The batch's sequences go in up to eight
    groups (at least four sequences each when the rank holds more than 16, else
    groups of one or two so that at least four are in flight), each with its
    own page pool: group
    i's host-to-device copies (one stream) overlap group i-1's attention call
    (torch's current stream) and group i-2's read-back (a third stream), so
    the step costs about the PCIe time of its bytes rather than the sum of
    copies and compute.
    """
    from minicpm_b200 import iluvatar_attention

    os.environ["ILUVATAR_USE_OPTIMIZED"] = "1"
    os.environ["ILUVATAR_SPLIT_KV"] = "1"
    os.environ["ILUVATAR_SPLIT_KV_DECODE"] = "1"  # a group of decode rows stays on the sm_100a kernels
    if splits:
        os.environ["ILUVATAR_NUM_SPLITS"] = str(splits)
    dev = out.device
    nseq = len(batch.query_lens)
    if nseq > 4 * E2E_MIN_SEQS_PER_GROUP:
        n_groups = min(E2E_MAX_GROUPS, nseq // E2E_MIN_SEQS_PER_GROUP)
    else:
        n_groups = min(nseq, max(E2E_MIN_GROUPS, nseq // 2), E2E_MAX_GROUPS)
    n_groups = max(1, n_groups)
    parts = split_into_groups(batch, n_groups)
    keys = ("q", "kv_cache", "block_table", "cu_seqlens_q", "seqused_k")
    host = [{k: getattr(p, k).pin_memory() for k in keys} for p in parts]
    host_out = [torch.empty(p.q.shape, dtype=p.q.dtype).pin_memory() for p in parts]
    dbuf = [{k: torch.empty(h[k].shape, dtype=h[k].dtype, device=dev) for k in keys} for h in host]
    dout = [torch.empty(p.q.shape, dtype=p.q.dtype, device=dev) for p in parts]
    h2d = sum(t.numel() * t.element_size() for h in host for t in h.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in parts]
    ev_done = [torch.cuda.Event() for _ in parts]
    ev_out = [torch.cuda.Event() for _ in parts]
    for i in range(len(parts)):
        ev_done[i].record(stream)
        ev_out[i].record(stream)

    def e2e_step():
        for i, p in enumerate(parts):
            h2d_s.wait_event(ev_done[i])  # the previous step's call has finished reading these buffers
            with torch.cuda.stream(h2d_s):
                for k in keys:
                    dbuf[i][k].copy_(host[i][k], non_blocking=True)
                ev_in[i].record(h2d_s)
            stream.wait_event(ev_in[i])
            stream.wait_event(ev_out[i])  # the previous step's read-back of dout[i] is done
            d = dbuf[i]
            iluvatar_attention(d["q"], d["kv_cache"], d["kv_cache"], dout[i], d["cu_seqlens_q"], p.max_seqlen_q,
                               d["seqused_k"], p.max_seqlen_k, p.softmax_scale, causal=True,
                               block_table=d["block_table"])
            ev_done[i].record(stream)
            d2h_s.wait_event(ev_done[i])
            with torch.cuda.stream(d2h_s):
                host_out[i].copy_(dout[i], non_blocking=True)
                ev_out[i].record(d2h_s)
        stream.wait_stream(d2h_s)

    for _ in range(max(1, min(args.warmup, 2))):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    h2d_s.wait_event(s)
    d2h_s.wait_event(s)
    for _ in range(args.steps):
        e2e_step()
    e.record(stream)
    e.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(s.elapsed_time(e), world)
    got = torch.cat(host_out) if host_out else torch.empty_like(out.cpu())
    want = out.cpu()
    identical = bool(torch.equal(got, want))
    if not identical:
        diff = (got.float() - want.float()).abs()
        assert diff.max().item() <= 2e-2 and diff.mean().item() <= 1e-3, "e2e output differs from the device-resident run"
    return {"value": total_flops * args.steps / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(sum_over_ranks(float(h2d), world)),
            "d2h_bytes_per_step": int(sum_over_ranks(float(d2h), world)),
            "ms_per_step": e2e_ms / args.steps,
            "tokens_per_s": total_tokens * args.steps / (e2e_ms * 1e-3),
            "api": "iluvatar_attention, one call per sequence group",
            "groups": len(parts), "overlap": "H2D of group i | attention of group i-1 | D2H of group i-2",
            "bit_identical_to_device_run": identical}


# --------------------------------------------------------------------- attention bench
def attention_run(workload: str, splits: int, steps: int, warmup: int, world: int, rank: int, local: int,
                  num_seqs: int = 0, graph: bool = False, clocks: bool = True, kv_quant: str = "none") -> dict:
    """Device-resident timing of ``steps`` back-to-back calls on this rank's shard.

    Barrier + synchronize on both sides of the timed region, CUDA events on the
    launching stream, the slowest rank's time.  Returns the whole-job figures
    and this rank's per-launch times.
    """
    from minicpm_b200 import paged_split_kv_attention
    from minicpm_b200.split_kv_paged import choose_num_splits
    from minicpm_b200.workloads import attention_kv_bytes
    from oracle import causal_flops  # FLOP formula of the reference harness (no compute)

    dev = torch.device("cuda", local)
    batch, all_q, all_kv = build_local_batch(workload, world, rank, num_seqs)
    local_flops = causal_flops(batch.query_lens, batch.kv_lens, 16, HEAD_DIM)
    local_bytes = attention_kv_bytes(batch.query_lens, batch.kv_lens, head_dim=HEAD_DIM)
    total_bytes = sum_over_ranks(float(local_bytes), world)
    total_flops = sum_over_ranks(float(local_flops), world)
    g = batch.to(dev)
    out = torch.empty_like(g.q)
    resolved = splits or choose_num_splits(g.total_q, len(batch.query_lens), 16, 2, batch.max_seqlen_k)

    def step():
        paged_split_kv_attention(g.q, g.kv_cache[:, 0], g.kv_cache[:, 1], out, g.block_table, g.seqused_k,
                                 g.cu_seqlens_q, g.max_seqlen_q, g.max_seqlen_k, g.softmax_scale, num_splits=splits)

    if kv_quant == "fp8":
        # The same pages as an fp8 e4m3 cache with per-tensor scales: each call
        # dequantises the pages it references, then runs the same kernel.
        from minicpm_b200 import unified_attention_optimized

        ks = torch.tensor([0.02], device=dev)
        vs = torch.tensor([0.02], device=dev)
        kc8 = (g.kv_cache[:, 0].float() / ks).to(torch.float8_e4m3fn)
        vc8 = (g.kv_cache[:, 1].float() / vs).to(torch.float8_e4m3fn)

        def step():  # noqa: F811
            unified_attention_optimized(g.q, kc8, vc8, out, g.block_table, g.seqused_k, g.cu_seqlens_q, g.max_seqlen_q,
                                        g.max_seqlen_k, g.softmax_scale, causal=True, num_splits_override=splits or None,
                                        kv_quant_mode=1, k_descale=ks, v_descale=vs)

    for _ in range(max(warmup, 1)):
        step()
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    if graph:
        # The K calls captured in one CUDA graph (as a serving engine replays
        # its decode steps) and replayed once inside the events.
        gstream = torch.cuda.Stream(device=dev)
        gstream.wait_stream(stream)
        cuda_graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(gstream):
            with torch.cuda.graph(cuda_graph, stream=gstream):
                for _ in range(steps):
                    step()
        stream.wait_stream(gstream)
        cuda_graph.replay()
        torch.cuda.synchronize(dev)
        barrier(world)
    sampler = ClockSampler(dev.index) if clocks else None
    if sampler:
        sampler.__enter__()
    try:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        start.record(stream)
        if graph:
            cuda_graph.replay()
        else:
            for s, e in evs:
                s.record(stream)
                step()
                e.record(stream)
        end.record(stream)
        end.synchronize()
    finally:
        if sampler:
            sampler.__exit__(None, None, None)
    barrier(world)
    elapsed_ms = start.elapsed_time(end)
    if graph:
        per_launch = [elapsed_ms / steps] * steps
        del cuda_graph
    else:
        per_launch = [s.elapsed_time(e) for s, e in evs]
    max_ms = max_over_ranks(elapsed_ms, world)
    rank_ms = gather_over_ranks(elapsed_ms, world)
    return {
        "batch": batch, "g": g, "out": out, "stream": stream, "resolved": resolved,
        "local_flops": local_flops, "local_bytes": local_bytes, "total_flops": total_flops,
        "total_bytes": total_bytes, "total_tokens": sum(all_q), "all_q": all_q,
        "max_ms": max_ms, "rank_ms": rank_ms, "per_launch": per_launch, "launch_ms": statistics.mean(per_launch),
        "value": total_flops * steps / (max_ms * 1e-3) / 1e12,
        "tokens_per_s": sum(all_q) * steps / (max_ms * 1e-3),
        "clocks": sampler.summary() if sampler else None,
    }


def traffic_per_launch(workload: str):
    """DRAM bytes per launch from the committed ncu summary of this workload, if any."""
    tfile = ROOT / "profiles" / f"paged_attn_fwd_{workload}.traffic.json"
    if tfile.exists():
        try:
            return json.loads(tfile.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


def sub_benchmarks(args, world, rank, local) -> dict:
    """The rest of the metric, measured in the same run as the headline.

    * the 4K chunked-prefill config at S = auto / 4 / 8 (TFLOP/s, sharded like
      the headline; S is the most splits a query unit gets), and at S = 4 with
      every query unit split (``_uniform``, the reference's rule);
    * the mixed 256-sequence batch (half decode rows), LPT-sharded over the
      ranks (TFLOP/s);
    * the RoPE + KV-cache write at rotary_dim 64 / 128 x NeoX / interleaved
      and the Split-KV combine at S = 4 (GB/s per GPU; every rank runs its own
      replica, the value is the sum over ranks).

    Each entry carries its roofline fraction against the measured peaks.
    """
    peaks, kind = measured_peaks()
    steps, warmup = max(5, args.steps // 2), 3
    subs = {}
    sampler = ClockSampler(local)
    sampler.__enter__()
    try:
        for workload, splits, uniform in (("chunked_prefill_4k", 0, False), ("chunked_prefill_4k", 4, False),
                                          ("chunked_prefill_4k", 8, False), ("chunked_prefill_4k", 4, True),
                                          ("mixed_256", 0, False)):
            if uniform:  # every query unit split `splits` ways: the reference's rule, for comparison
                os.environ["B200_ATTN_SPLIT_UNIFORM"] = "1"
            try:
                r = attention_run(workload, splits, steps, warmup, world, rank, local, clocks=False)
                verify = None
                if workload == "mixed_256" and world > 1 and not args.no_verify:
                    verify = verify_sharded(workload, 0, r["batch"], r["out"], world, rank, splits)
            finally:
                os.environ.pop("B200_ATTN_SPLIT_UNIFORM", None)
            achieved = r["local_flops"] / (r["launch_ms"] * 1e-3) / 1e12
            name = (f"{workload}_S{splits}" if splits else f"{workload}_auto") + ("_uniform" if uniform else "")
            subs[name] = {
                "value": r["value"], "unit": "TFLOP/s", "ms_per_step": r["max_ms"] / steps, "steps": steps,
                "gpu_launches": steps * (2 + (1 if r["resolved"] > 1 else 0)),
                "tokens_per_s": r["tokens_per_s"], "num_splits": r["resolved"], "causal_flops": r["total_flops"],
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": achieved / peaks["bf16_tflops"],
                             "traffic": traffic_per_launch(workload) if splits == 0 else None,
                             "peak_kind": f"bf16_tflops (burst) of {kind}", "per_launch_ms": r["launch_ms"]},
            }
            if world > 1:
                subs[name]["rank_spread"] = rank_spread(r["rank_ms"], steps)
            if verify:
                subs[name]["verify"] = verify
            del r
            torch.cuda.empty_cache()
        for rd in (64, 128):
            for neox in (True, False):
                n = max(10, args.steps)
                r = rope_run(rd, neox, False, "auto", n, warmup, local, world, clocks=False)
                subs[f"rope_16384_rd{rd}_{'neox' if neox else 'interleaved'}"] = {
                    "value": r["gbs"] * world, "unit": "GB/s", "us_per_launch": r["ms"] * 1e3, "gpu_launches": n,
                    "algorithmic_bytes": r["nbytes"], "timing": "CUDA graph of the timed launches",
                    "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                 "frac": r["gbs"] / peaks["hbm_gbs"], "traffic": None, "peak_kind": kind},
                }
                del r
        n = max(10, args.steps)
        r = combine_run(4, n, warmup, local, world, clocks=False)
        subs["split_combine_4k_S4"] = {
            "value": r["gbs"] * world, "unit": "GB/s", "us_per_launch": r["ms"] * 1e3, "gpu_launches": n,
            "algorithmic_bytes": r["nbytes"], "timing": "CUDA graph of the timed launches",
            "roofline": {"bound": "hbm", "achieved": r["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": r["gbs"] / peaks["hbm_gbs"], "traffic": None, "peak_kind": kind},
        }
        del r
        torch.cuda.empty_cache()
    finally:
        sampler.__exit__(None, None, None)
    subs["clocks"] = sampler.summary()
    return subs


def attention_bench(args, world, rank, local):
    from minicpm_b200.workloads import attention_kv_bytes

    decode = args.workload.startswith("decode")
    r = attention_run(args.workload, args.splits, args.steps, args.warmup, world, rank, local, args.num_seqs,
                      graph=args.graph, kv_quant=args.kv_quant)
    batch, out, stream = r["batch"], r["out"], r["stream"]
    max_ms, total_flops, total_tokens = r["max_ms"], r["total_flops"], r["total_tokens"]

    # e2e: public operator API, host buffers, copies inside the timed region.
    e2e = None
    if not args.no_e2e:
        e2e = e2e_pipelined(args, batch, out, args.splits, stream, world, total_flops, total_tokens)

    verify = None
    if args.verify or (world > 1 and not args.no_verify):
        verify = verify_sharded(args.workload, args.num_seqs, batch, out, world, rank, args.splits)

    subs = None
    if (args.workload == "chunked_prefill_16k" and not args.no_sub and not args.num_seqs and HEAD_DIM == 128
            and args.kv_quant == "none"):
        del r["g"], r["out"]
        out = None
        torch.cuda.empty_cache()
        subs = sub_benchmarks(args, world, rank, local)

    if rank != 0:
        return
    peaks, peak_kind = measured_peaks()
    launch_ms = r["launch_ms"]
    achieved = r["local_flops"] / (launch_ms * 1e-3) / 1e12
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        run, flops_s, desc = cpu_sample_flops(batch, 512)
        run()
        ts = time_cpu(run, 2)
        if decode:
            sample_bytes = attention_kv_bytes([1], [batch.kv_lens[0]])
            cpu = {"value": sample_bytes / statistics.mean(ts) / 1e9, "unit": "GB/s",
                   "cores": torch.get_num_threads(), "kind": "port", "sample": desc}
        else:
            cpu = {"value": flops_s / statistics.mean(ts) / 1e12, "unit": "TFLOP/s",
                   "cores": torch.get_num_threads(), "kind": "port", "sample": desc}
    config = attention_config(args.workload, world, args.splits, args.num_seqs)
    if args.kv_quant != "none":
        config["kv_cache"] = f"{args.kv_quant} per-tensor (pages dequantised each call)"
    line = {
        "metric": METRIC,
        "value": r["value"],
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": max_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, random-permuted page table)",
        "tokens_per_s": r["tokens_per_s"],
        "tc_peak_frac": r["value"] / world / peaks["bf16_tflops"],
        "config": config,
        "timing": "one CUDA graph of the K calls" if args.graph else "K calls launched from Python",
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"], "traffic": traffic_per_launch(args.workload),
                     "peak_kind": f"bf16_tflops (burst) of {peak_kind}",
                     "per_launch_ms": launch_ms, "launch": "schedule + attention kernels of one call"},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": r["clocks"],
        "gpu_launches": args.steps * (2 + (1 if r["resolved"] > 1 else 0)),
    }
    if world > 1:
        line["rank0_ms_per_step"] = sum(r["per_launch"]) / args.steps
        line["rank_spread"] = rank_spread(r["rank_ms"], args.steps)
    if verify:
        line["verify"] = verify
    if decode:
        # Decode streams every K/V row once for a handful of query rows: the
        # bound is HBM, and the metric is the bytes moved per second.
        total_bytes, local_bytes = r["total_bytes"], r["local_bytes"]
        gbs = total_bytes * args.steps / (max_ms * 1e-3) / 1e9
        achieved_gbs = local_bytes / (launch_ms * 1e-3) / 1e9
        line.update({
            "metric": "paged decode attention GB/s (K/V streamed once)", "value": gbs, "unit": "GB/s",
            "tc_peak_frac": None, "decode_tokens_per_s": r["tokens_per_s"],
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved_gbs / peaks["hbm_gbs"], "traffic": None, "peak_kind": peak_kind,
                         "per_launch_ms": launch_ms, "launch": "schedule + attention (+ combine) kernels of one call"},
        })
        line["config"]["algorithmic_bytes"] = total_bytes
        if e2e:
            e2e["value"] = total_bytes * args.steps / (e2e["ms_per_step"] * args.steps * 1e-3) / 1e9
            e2e["unit"] = "GB/s"
    if subs:
        line["sub"] = subs
        line["gpu_launches"] += sum(v.get("gpu_launches", 0) for v in subs.values() if isinstance(v, dict))
    print(json.dumps(line), flush=True)


def main():
    global HEAD_DIM
    args = parse_args()
    HEAD_DIM = args.head_dim
    if args.impl == "reference":
        # Rank 0 alone times the host-core implementation; other ranks exit at once.
        if int(os.environ.get("RANK", "0")) == 0:
            reference_arm(args, int(os.environ.get("WORLD_SIZE", "1")), 0)
        return
    world, rank, local = dist_setup(args)
    try:
        if args.workload == "rope_16384":
            rope_bench(args, world, rank, local)
        elif args.workload == "kv_write_16384":
            kv_write_bench(args, world, rank, local)
        elif args.workload == "split_combine_4k":
            combine_bench(args, world, rank, local)
        else:
            attention_bench(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
