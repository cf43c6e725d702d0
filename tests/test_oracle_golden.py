"""Pin the CPU oracle against vectors from the reference's own kernels.

The fixtures in ``tests/golden`` were produced by ``tests/golden/make_golden.py``
running the reference's Triton kernels under ``TRITON_INTERPRET=1``.  The
inputs are rebuilt here from the seeded generators and checked by sha256.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from minicpm_b200 import workloads
from oracle import (
    paged_attention_reference,
    rope_and_cache_reference,
    rotate_fp32,
    split_kv_partials_reference,
    split_kv_reduce_reference,
)

ATTN = ["small_a", "small_b", "small_c", "small_short_kv", "ref_case_1", "ref_case_2"]


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _load_attn(golden_dir, name):
    rec = dict(np.load(golden_dir / f"attn_{name}.npz"))
    heads, kv_heads, dim, pool = (int(x) for x in rec["dims"])
    batch = workloads.build_attention_batch(
        rec["query_lens"].tolist(), rec["kv_lens"].tolist(), seed=workloads.DEFAULT_SEED,
        num_q_heads=heads, num_kv_heads=kv_heads, head_dim=dim, pool_pages=pool or None,
        dtype=torch.bfloat16,
    )
    assert _sha(batch.q) == str(rec["sha_q"]), "input generator changed: regenerate the golden files"
    assert _sha(batch.kv_cache) == str(rec["sha_cache"])
    assert _sha(batch.block_table) == str(rec["sha_table"])
    return rec, batch


@pytest.mark.parametrize("name", ATTN)
def test_oracle_matches_reference_output(golden_dir, name):
    rec, b = _load_attn(golden_dir, name)
    got = paged_attention_reference(b.q, b.k_cache, b.v_cache, b.block_table, b.cu_seqlens_q, b.seqused_k, b.softmax_scale)
    for s in rec["splits"].tolist():
        want = torch.from_numpy(rec[f"out_s{s}"])
        err = (got - want).abs().max().item()
        assert err < 2e-5, (name, s, err)


@pytest.mark.parametrize("name", [n for n in ATTN if n.startswith("small")])
def test_oracle_split_partials_match_reference(golden_dir, name):
    rec, b = _load_attn(golden_dir, name)
    for s in rec["splits"].tolist():
        o, m, l = split_kv_partials_reference(b.q, b.k_cache, b.v_cache, b.block_table, b.cu_seqlens_q, b.seqused_k, b.softmax_scale, s)
        want_m = torch.from_numpy(rec[f"m_split_s{s}"])
        want_l = torch.from_numpy(rec[f"l_split_s{s}"])
        want_o = torch.from_numpy(rec[f"o_split_s{s}"])
        # Empty splits: exactly -inf / 0 in both.
        assert torch.equal(torch.isinf(m), torch.isinf(want_m)), (name, s)
        assert torch.equal(l == 0, want_l == 0), (name, s)
        fin = torch.isfinite(want_m)
        assert (m[fin] - want_m[fin]).abs().max().item() < 1e-5
        assert ((l - want_l).abs() / want_l.clamp(min=1)).max().item() < 1e-5
        assert (o - want_o).abs().max().item() < 2e-5


@pytest.mark.parametrize("name", [n for n in ATTN if n.startswith("small")])
def test_oracle_reduce_matches_reference(golden_dir, name):
    rec, _ = _load_attn(golden_dir, name)
    for s in rec["splits"].tolist():
        red = split_kv_reduce_reference(
            torch.from_numpy(rec[f"o_split_s{s}"]), torch.from_numpy(rec[f"m_split_s{s}"]), torch.from_numpy(rec[f"l_split_s{s}"])
        )
        want = torch.from_numpy(rec[f"reduce_s{s}"])
        assert (red - want).abs().max().item() < 1e-6


def _rope_inputs(is_neox, rd):
    g = torch.Generator().manual_seed(workloads.DEFAULT_SEED + int(is_neox) * 100 + rd)
    query = torch.randn(9, 16, 128, generator=g).to(torch.bfloat16)
    key = torch.randn(9, 2, 128, generator=g).to(torch.bfloat16)
    value = torch.randn(9, 2, 128, generator=g).to(torch.bfloat16)
    positions = torch.tensor([0, 3, 17, 31, 63, 127, 255, 511, 1023], dtype=torch.int32)
    angles = torch.randn(2048, rd // 2, generator=g)
    cos_sin = torch.cat((angles.cos(), angles.sin()), dim=-1).to(torch.bfloat16)
    slots = torch.tensor([0, 17, 34, 51, 68, 85, 102, 119, -1], dtype=torch.int32)
    kc = torch.full((8, 16, 2, 128), 7.0, dtype=torch.bfloat16)
    vc = torch.full_like(kc, -7.0)
    return query, key, value, positions, cos_sin, slots, kc, vc


def _truncate_to_bf16_bits(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 by dropping the low 16 bits (round toward zero), as int16."""
    return (x.contiguous().view(torch.int32) >> 16).to(torch.int16)


@pytest.mark.parametrize("is_neox", [True, False])
@pytest.mark.parametrize("rd", [64, 128])
def test_oracle_rope_bit_exact_vs_reference(golden_dir, is_neox, rd):
    """The oracle's fp32 rotation equals the reference kernel's, bit for bit.

    The Triton CPU interpreter casts fp32 to bf16 by truncation, while the GPU
    store (and torch) round to nearest even.  So the pin is: the oracle's fp32
    result, truncated, equals the interpreter's bytes exactly; and the
    oracle's rounded result is within one bf16 ulp of them.
    """
    rec = np.load(golden_dir / "rope_reference_cases.npz")
    tag = f"{'neox' if is_neox else 'gptj'}_{rd}_"
    query, key, value, positions, cos_sin, slots, kc, vc = _rope_inputs(is_neox, rd)
    assert _sha(query) == str(rec[tag + "sha_query"])
    assert _sha(key) == str(rec[tag + "sha_key"])
    assert _sha(value) == str(rec[tag + "sha_value"])
    assert _sha(cos_sin) == str(rec[tag + "sha_cos_sin"])
    want_q = torch.from_numpy(rec[tag + "query_out"])
    want_k = torch.from_numpy(rec[tag + "key_cache_out"])
    want_v = torch.from_numpy(rec[tag + "value_cache_out"])

    q32 = rotate_fp32(query, cos_sin, positions, is_neox, rd)
    k32 = rotate_fp32(key, cos_sin, positions, is_neox, rd)
    assert torch.equal(_truncate_to_bf16_bits(q32), want_q)
    kc_trunc = kc.view(torch.int16).clone()
    for t, slot in enumerate(slots.tolist()):
        if slot >= 0:
            kc_trunc[slot // 16, slot % 16] = _truncate_to_bf16_bits(k32[t])
    assert torch.equal(kc_trunc, want_k)

    q_out, k_out, v_out = rope_and_cache_reference(query, key, value, positions, cos_sin, is_neox, kc, vc, slots, rd)
    assert (q_out.float() - want_q.view(torch.bfloat16).float()).abs().max().item() <= 0.0625
    ulps = (q_out.view(torch.int16).int() - want_q.int()).abs().max().item()
    assert ulps <= 1
    assert torch.equal(v_out.view(torch.int16), want_v)  # V is a copy: exact
    # The negative slot leaves the sentinel in place (tests/test_rope_kv_cache.py:70).
    assert torch.equal(k_out[-1, -1], torch.full_like(k_out[-1, -1], 7))
