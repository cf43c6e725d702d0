"""Parity of the sm_100a RoPE + paged KV-cache write against the oracle (GPU).

The reference's four cases (tests/test_rope_kv_cache.py:35-86), the golden
bytes of the reference kernel, and the 16384-token workload at rotary_dim
64/128 x NeoX/interleaved.  Bar: Q and cached K bit-exact with the oracle
(which rounds like the GPU store), cache placement and V exact, untouched
slots keep their sentinel, negative slots write nothing.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from minicpm_b200 import _lib, fused_rope_and_cache
from minicpm_b200.workloads import build_rope_batch
from oracle import rope_and_cache_reference

pytestmark = pytest.mark.gpu


def _run(b, **kw):
    g = b.to("cuda")
    fused_rope_and_cache(
        g.query, g.key, g.value, g.positions, g.cos_sin_cache, g.is_neox, g.key_cache, g.value_cache,
        g.slot_mapping, rotary_dim=kw.get("rotary_dim", g.rotary_dim),
    )
    torch.cuda.synchronize()
    return g


def _check_exact(b, g):
    q_want, kc_want, vc_want = rope_and_cache_reference(
        b.query, b.key, b.value, b.positions, b.cos_sin_cache, b.is_neox, b.key_cache, b.value_cache,
        b.slot_mapping, b.rotary_dim,
    )
    assert torch.equal(g.query.cpu().view(torch.int16), q_want.view(torch.int16))
    assert torch.equal(g.key_cache.cpu().view(torch.int16), kc_want.view(torch.int16))
    assert torch.equal(g.value_cache.cpu().view(torch.int16), vc_want.view(torch.int16))
    # key/value inputs untouched
    assert torch.equal(g.key.cpu(), b.key) and torch.equal(g.value.cpu(), b.value)


def _reference_case(is_neox, rd):
    gen = torch.Generator().manual_seed(20260928 + int(is_neox) * 100 + rd)
    query = torch.randn(9, 16, 128, generator=gen).to(torch.bfloat16)
    key = torch.randn(9, 2, 128, generator=gen).to(torch.bfloat16)
    value = torch.randn(9, 2, 128, generator=gen).to(torch.bfloat16)
    positions = torch.tensor([0, 3, 17, 31, 63, 127, 255, 511, 1023], dtype=torch.int32)
    angles = torch.randn(2048, rd // 2, generator=gen)
    cos_sin = torch.cat((angles.cos(), angles.sin()), dim=-1).to(torch.bfloat16)
    slots = torch.tensor([0, 17, 34, 51, 68, 85, 102, 119, -1], dtype=torch.int32)
    kc = torch.full((8, 16, 2, 128), 7.0, dtype=torch.bfloat16)
    vc = torch.full_like(kc, -7.0)
    from minicpm_b200.workloads import RopeBatch

    return RopeBatch(query, key, value, positions, cos_sin, kc, vc, slots, is_neox, rd)


@pytest.mark.parametrize("is_neox", [True, False])
@pytest.mark.parametrize("rd", [64, 128])
def test_reference_cases(golden_dir, is_neox, rd):
    b = _reference_case(is_neox, rd)
    g = _run(b)
    _check_exact(b, g)
    # The negative slot leaves the sentinel (tests/test_rope_kv_cache.py:70).
    assert torch.equal(g.key_cache[-1, -1].cpu(), torch.full((2, 128), 7.0, dtype=torch.bfloat16))
    # Against the reference kernel's own bytes: within one bf16 ulp (the CPU
    # interpreter that produced them truncates where the GPU rounds).
    rec = np.load(golden_dir / "rope_reference_cases.npz")
    tag = f"{'neox' if is_neox else 'gptj'}_{rd}_"
    for name, t in (("query_out", g.query), ("key_cache_out", g.key_cache), ("value_cache_out", g.value_cache)):
        want = torch.from_numpy(rec[tag + name]).int()
        assert (t.cpu().view(torch.int16).int() - want).abs().max().item() <= 1, name
    assert _lib.device_error() == _lib.DEVERR_NONE


@pytest.mark.parametrize("is_neox", [True, False])
@pytest.mark.parametrize("rd", [64, 128])
def test_full_16384_tokens(is_neox, rd):
    b = build_rope_batch(16384, rotary_dim=rd, is_neox=is_neox)
    g = _run(b)
    _check_exact(b, g)
    # Every slot not in the mapping still holds its sentinel.
    written = torch.zeros(4096 * 16, dtype=torch.bool)
    written[b.slot_mapping.long()] = True
    kc = g.key_cache.cpu().reshape(4096 * 16, 2, 128)
    assert (kc[~written] == 7).all() and (g.value_cache.cpu().reshape(4096 * 16, 2, 128)[~written] == -7).all()
    assert _lib.device_error() == _lib.DEVERR_NONE


@pytest.mark.parametrize("pos_dtype,slot_dtype", [(torch.int32, torch.int32), (torch.int64, torch.int32), (torch.int32, torch.int64)])
def test_index_dtypes_and_negative_slots(pos_dtype, slot_dtype):
    b = build_rope_batch(1000, rotary_dim=128, is_neox=True, pos_dtype=pos_dtype, slot_dtype=slot_dtype)
    b.slot_mapping[::7] = -1
    g = _run(b)
    _check_exact(b, g)


@pytest.mark.parametrize("head_dim,rd", [(64, 64), (256, 128), (128, 32)])
def test_other_head_dims(head_dim, rd):
    for neox in (True, False):
        b = build_rope_batch(300, rotary_dim=rd, is_neox=neox, head_dim=head_dim, num_blocks=64)
        _check_exact(b, _run(b))


def test_fp16_and_fp32_cos_sin():
    b = build_rope_batch(500, rotary_dim=64, is_neox=False, dtype=torch.float16)
    _check_exact(b, _run(b))
    b = build_rope_batch(500, rotary_dim=128, is_neox=True)
    b.cos_sin_cache = b.cos_sin_cache.float()
    _check_exact(b, _run(b))


def test_strided_views_use_scalar_or_vector_paths():
    # q/k/v as views into one fused qkv buffer (vector path), and a query
    # with a non-unit head-dim stride (element path).
    b = build_rope_batch(257, rotary_dim=128, is_neox=True)
    qkv = torch.cat([b.query, b.key, b.value], dim=1)  # [T, 20, 128]
    g_qkv = qkv.cuda()
    q, k, v = g_qkv[:, :16], g_qkv[:, 16:18], g_qkv[:, 18:20]
    kc, vc = b.key_cache.cuda(), b.value_cache.cuda()
    fused_rope_and_cache(q, k, v, b.positions.cuda(), b.cos_sin_cache.cuda(), True, kc, vc, b.slot_mapping.cuda())
    q_want, kc_want, vc_want = rope_and_cache_reference(
        b.query, b.key, b.value, b.positions, b.cos_sin_cache, True, b.key_cache, b.value_cache, b.slot_mapping
    )
    assert torch.equal(q.cpu(), q_want) and torch.equal(kc.cpu(), kc_want) and torch.equal(vc.cpu(), vc_want)

    qt = b.query.transpose(1, 2).contiguous().cuda().transpose(1, 2)  # d stride = 16
    kc2, vc2 = b.key_cache.cuda(), b.value_cache.cuda()
    fused_rope_and_cache(qt, b.key.cuda(), b.value.cuda(), b.positions.cuda(), b.cos_sin_cache.cuda(), True, kc2, vc2,
                         b.slot_mapping.cuda())
    assert torch.equal(qt.cpu(), q_want) and torch.equal(kc2.cpu(), kc_want)


def test_out_of_range_slot_is_skipped_and_reported():
    b = build_rope_batch(64, rotary_dim=128, is_neox=True, num_blocks=8)
    b.slot_mapping[3] = 8 * 16 + 5  # one past the end of the cache
    g = _run(b)
    assert _lib.device_error() == _lib.DEVERR_SLOT_RANGE
    assert _lib.device_error() == _lib.DEVERR_NONE  # read-and-clear
    keep = torch.ones(64, dtype=torch.bool)
    keep[3] = False
    b2 = b.clone()
    b2.slot_mapping[3] = -1
    q_want, kc_want, _ = rope_and_cache_reference(
        b2.query, b2.key, b2.value, b2.positions, b2.cos_sin_cache, True, b2.key_cache, b2.value_cache, b2.slot_mapping
    )
    assert torch.equal(g.query.cpu(), q_want) and torch.equal(g.key_cache.cpu(), kc_want)
