"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own Triton kernels on the CPU under ``TRITON_INTERPRET=1``
(``kernels/triton_split_kv_paged.py`` and ``kernels/triton_rope_kv_cache.py``
of the reference project) on small seeded inputs and stores their outputs.

* Attention: fp32 inputs whose values are bf16-representable (the interpreter
  gives invalid attention output for bf16 inputs, so the golden runs use fp32
  tensors holding the same values the GPU tests use in bf16).  Stored: the
  final output of ``paged_split_kv_attention`` and, for the small-head cases,
  the per-split partials of ``_split_kv_forward`` and the output of
  ``_split_kv_reduce`` on those partials.
* RoPE: the reference test's four cases (9 tokens at fixed positions, fixed
  slots including ``-1``, sentinel-filled caches), run in bf16.

Inputs are not stored: the tests rebuild them from the seeded CPU generators
in ``minicpm_b200.workloads`` and check their sha256 against the value
recorded here, so a changed generator fails loudly instead of silently.

Usage (only where the reference project is mounted)::

    python tests/golden/make_golden.py --reference <checkout of the reference project>
"""

from __future__ import annotations

import argparse
import hashlib
import math
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "minicpm-attention-optimization-iluvatar_b200"))

from minicpm_b200 import workloads  # noqa: E402

# name, heads, kv_heads, head_dim, query_lens, kv_lens, pool, splits, store partials
ATTN_CASES = [
    ("small_a", 4, 2, 64, [5, 1, 9], [25, 48, 9], 0, (2, 4, 8), True),
    ("small_b", 4, 2, 64, [33, 16, 1, 7], [33, 100, 200, 7], 40, (2, 4, 8), True),
    ("small_c", 8, 1, 64, [20, 3], [70, 3], 0, (4,), True),
    ("small_short_kv", 4, 2, 64, [6, 2], [6, 64], 0, (8, 16), True),
    ("ref_case_1", 16, 2, 128, [1, 17, 65], [128, 128, 128], 0, (4,), False),
    ("ref_case_2", 16, 2, 128, [31, 1, 13], [31, 256, 1014], 0, (8,), False),
]

ROPE_POSITIONS = [0, 3, 17, 31, 63, 127, 255, 511, 1023]
ROPE_SLOTS = [0, 17, 34, 51, 68, 85, 102, 119, -1]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def attn_case(ref, name, heads, kv_heads, dim, qlens, kvlens, pool, splits, partials):
    from kernels.triton_split_kv_paged import _split_kv_forward, _split_kv_reduce, paged_split_kv_attention

    batch = workloads.build_attention_batch(
        qlens, kvlens, seed=workloads.DEFAULT_SEED, num_q_heads=heads, num_kv_heads=kv_heads,
        head_dim=dim, pool_pages=pool or None, dtype=torch.bfloat16,
    )
    q = batch.q.float()
    cache = batch.kv_cache.float()
    k, v = cache[:, 0], cache[:, 1]
    rec = {
        "query_lens": np.array(qlens, np.int64),
        "kv_lens": np.array(kvlens, np.int64),
        "dims": np.array([heads, kv_heads, dim, pool], np.int64),
        "splits": np.array(splits, np.int64),
        "sha_q": np.array(sha(batch.q)),
        "sha_cache": np.array(sha(batch.kv_cache)),
        "sha_table": np.array(sha(batch.block_table)),
    }
    for s in splits:
        out = torch.empty_like(q)
        paged_split_kv_attention(
            q, k, v, out, batch.block_table, batch.seqused_k, batch.cu_seqlens_q,
            batch.max_seqlen_q, batch.max_seqlen_k, batch.softmax_scale,
            num_splits=s, block_m=16, block_n=16,
        )
        rec[f"out_s{s}"] = out.numpy().astype(np.float32)
        if not partials:
            continue
        # The forward and the reduce launched exactly as the reference's host
        # wrapper launches them (kernels/triton_split_kv_paged.py:283-360),
        # keeping the intermediate buffers.
        block_m, block_n = 16, 16
        cu = batch.cu_seqlens_q
        per = (cu[1:] - cu[:-1] + block_m - 1) // block_m
        total_blocks = int(per.sum())
        ids = torch.arange(len(qlens), dtype=torch.int32)
        block_batch = torch.repeat_interleave(ids, per)
        starts = torch.cumsum(per, 0) - per
        block_q = torch.arange(total_blocks, dtype=torch.int32) - torch.repeat_interleave(starts, per)
        max_split_blocks = math.ceil(batch.max_seqlen_k / s / block_n) + 1
        o_s = torch.zeros(s, q.shape[0], heads, dim)
        m_s = torch.full((s, q.shape[0], heads), -float("inf"))
        l_s = torch.zeros_like(m_s)
        _split_kv_forward[(total_blocks, heads, s)](
            block_batch, block_q, q, k, v, batch.block_table, cu, batch.seqused_k,
            o_s, m_s, l_s,
            q.stride(0), q.stride(1), q.stride(2),
            k.stride(0), k.stride(1), k.stride(2), k.stride(3),
            v.stride(0), v.stride(1), v.stride(2), v.stride(3),
            batch.block_table.stride(0),
            o_s.stride(0), o_s.stride(1), o_s.stride(2), o_s.stride(3),
            m_s.stride(0), m_s.stride(1), m_s.stride(2),
            l_s.stride(0), l_s.stride(1), l_s.stride(2),
            num_q_heads=heads, num_kv_heads=kv_heads, head_dim=dim, block_size=16,
            num_splits=s, max_kv_blocks_per_split=max_split_blocks,
            BLOCK_M=block_m, BLOCK_N=block_n, BLOCK_D=dim, scale=batch.softmax_scale,
        )
        red = torch.empty_like(q)
        _split_kv_reduce[(total_blocks, heads)](
            block_batch, block_q, o_s, m_s, l_s, red, cu,
            o_s.stride(0), o_s.stride(1), o_s.stride(2), o_s.stride(3),
            m_s.stride(0), m_s.stride(1), m_s.stride(2),
            l_s.stride(0), l_s.stride(1), l_s.stride(2),
            red.stride(0), red.stride(1), red.stride(2),
            num_q_heads=heads, num_splits=s, BLOCK_M=block_m, BLOCK_D=dim,
        )
        rec[f"o_split_s{s}"] = o_s.numpy()
        rec[f"m_split_s{s}"] = m_s.numpy()
        rec[f"l_split_s{s}"] = l_s.numpy()
        rec[f"reduce_s{s}"] = red.numpy()
    return rec


def rope_inputs(is_neox: bool, rotary_dim: int):
    """The reference test's RoPE case (tests/test_rope_kv_cache.py:35-47) on a CPU generator."""
    g = torch.Generator().manual_seed(workloads.DEFAULT_SEED + int(is_neox) * 100 + rotary_dim)
    tokens, q_heads, kv_heads, head_dim, block_size, blocks = 9, 16, 2, 128, 16, 8
    query = torch.randn(tokens, q_heads, head_dim, generator=g).to(torch.bfloat16)
    key = torch.randn(tokens, kv_heads, head_dim, generator=g).to(torch.bfloat16)
    value = torch.randn(tokens, kv_heads, head_dim, generator=g).to(torch.bfloat16)
    positions = torch.tensor(ROPE_POSITIONS, dtype=torch.int32)
    angles = torch.randn(2048, rotary_dim // 2, generator=g)
    cos_sin = torch.cat((angles.cos(), angles.sin()), dim=-1).to(torch.bfloat16)
    slots = torch.tensor(ROPE_SLOTS, dtype=torch.int32)
    key_cache = torch.full((blocks, block_size, kv_heads, head_dim), 7.0, dtype=torch.bfloat16)
    value_cache = torch.full_like(key_cache, -7.0)
    return query, key, value, positions, cos_sin, slots, key_cache, value_cache


def rope_case(is_neox: bool, rotary_dim: int):
    from kernels.triton_rope_kv_cache import fused_rope_and_cache

    query, key, value, positions, cos_sin, slots, key_cache, value_cache = rope_inputs(is_neox, rotary_dim)
    rec = {
        "sha_query": np.array(sha(query)),
        "sha_key": np.array(sha(key)),
        "sha_value": np.array(sha(value)),
        "sha_cos_sin": np.array(sha(cos_sin)),
    }
    fused_rope_and_cache(query, key, value, positions, cos_sin, is_neox, key_cache, value_cache, slots, rotary_dim=rotary_dim)
    rec["query_out"] = query.view(torch.int16).numpy()
    rec["key_cache_out"] = key_cache.view(torch.int16).numpy()
    rec["value_cache_out"] = value_cache.view(torch.int16).numpy()
    return rec


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MINICPM_REFERENCE_DIR"),
                    help="checkout of the reference project (or set MINICPM_REFERENCE_DIR)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or MINICPM_REFERENCE_DIR) must name the reference project's checkout")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    for case in ATTN_CASES:
        if args.only and args.only not in case[0]:
            continue
        rec = attn_case(args.reference, *case)
        np.savez_compressed(HERE / f"attn_{case[0]}.npz", **rec)
        print("wrote", case[0], flush=True)
    rope = {}
    for is_neox in (True, False):
        for rd in (64, 128):
            if args.only and args.only != "rope":
                continue
            for k, v in rope_case(is_neox, rd).items():
                rope[f"{'neox' if is_neox else 'gptj'}_{rd}_{k}"] = v
    if rope:
        np.savez_compressed(HERE / "rope_reference_cases.npz", **rope)
        print("wrote rope", flush=True)


if __name__ == "__main__":
    main()
