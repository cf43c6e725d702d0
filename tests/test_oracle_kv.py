"""Pin the KV-cache-write oracle: fp8 encoder, vLLM golden vectors, host validation.

* The fp8 encoder of the oracle is checked against torch's float8 conversion
  on every bf16 value and on two million random fp32 values (torch's
  conversion is non-saturating, so its input is clamped to the finite range
  first; a saturating round-to-nearest-even conversion equals that).
* The plain and int8 per-token-head cache writes of the oracle are checked
  against the output of vLLM's own Triton kernels, run under the Triton
  interpreter by ``tests/golden/make_kv_golden.py``.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from minicpm_b200 import kv_cache, workloads
from oracle import fp8_decode, fp8_encode, kv_write_reference, quantize_per_token_head

FP8 = {"e4m3": (torch.float8_e4m3fn, 448.0), "e5m2": (torch.float8_e5m2, 57344.0)}


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_encoder_matches_torch_on_every_bf16_value(fmt):
    td, mx = FP8[fmt]
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    finite = ~np.isnan(x)
    mine = fp8_encode(x, fmt)
    ref = torch.from_numpy(x.copy()).clamp(-mx, mx).to(td).view(torch.uint8).numpy()
    assert np.array_equal(mine[finite], ref[finite])
    # saturation: the largest finite value, never a NaN code, for |x| beyond it (infinities included)
    big = np.array([mx * 1.01, -mx * 4, np.inf, -np.inf, 1e30], np.float32)
    assert np.array_equal(fp8_decode(fp8_encode(big, fmt), fmt), np.clip(big, -mx, mx))


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_encoder_matches_torch_on_random_fp32(fmt):
    td, mx = FP8[fmt]
    rng = np.random.default_rng(7)
    y = (rng.standard_normal(2_000_000) * np.exp2(rng.integers(-30, 20, 2_000_000))).astype(np.float32)
    ref = torch.from_numpy(y).clamp(-mx, mx).to(td).view(torch.uint8).numpy()
    assert np.array_equal(fp8_encode(y, fmt), ref)
    codes = np.arange(256, dtype=np.uint8)
    dec, tdec = fp8_decode(codes, fmt), torch.from_numpy(codes).view(td).float().numpy()
    assert np.array_equal(np.isnan(dec), np.isnan(tdec))
    assert np.array_equal(dec[~np.isnan(dec)], tdec[~np.isnan(tdec)])


def test_per_token_head_quantisation_edges():
    x = torch.zeros(3, 8)
    x[1, 3] = -5.0
    x[2] = torch.linspace(-1, 1, 8)
    codes, s = quantize_per_token_head(x, "int8")
    assert s[0] == np.float32(1e-6)  # all-zero head: the floor scale, codes zero
    assert not codes[0].any()
    assert codes[1, 3] == -127 and s[1] == np.float32(5.0) / np.float32(127.0)
    assert codes[2].max() == 127 and codes[2].min() == -127
    codes8, s8 = quantize_per_token_head(x, "e4m3")
    assert fp8_decode(codes8[1:2], "e4m3")[0, 3] == -448.0


def _golden_cases(golden_dir):
    z = np.load(golden_dir / "kv_write_vllm_cases.npz")
    names = sorted({k.split("__")[0] for k in z.keys()})
    return z, names


def test_oracle_matches_vllm_kernels(golden_dir):
    z, names = _golden_cases(golden_dir)
    assert len(names) == 5
    for name in names:
        rec = {k.split("__")[1]: z[k] for k in z.keys() if k.startswith(name + "__")}
        tokens, kh, d, blocks, pad = (int(v) for v in rec["dims"])
        dtype = getattr(torch, str(rec["dtype"]))
        kind = str(rec["kind"])
        b = workloads.build_kv_write_batch(
            tokens, kv_cache_dtype=kind, num_kv_heads=kh, head_dim=d, num_blocks=blocks, padding_tokens=pad, dtype=dtype
        )
        assert _sha(b.key) == str(rec["sha_key"]), f"{name}: input generator changed: regenerate the golden files"
        assert _sha(b.value) == str(rec["sha_value"]) and _sha(b.slot_mapping) == str(rec["sha_slots"])
        kc, vc = b.caches()
        ksc, vsc = (torch.zeros(kc.shape[:3]), torch.zeros(kc.shape[:3])) if kind != "auto" else (None, None)
        okc, ovc, oks, ovs = kv_write_reference(b.key, b.value, kc, vc, b.slot_mapping, kind, k_scale_cache=ksc, v_scale_cache=vsc)
        slots = b.slot_mapping.long()
        idx = torch.nonzero(slots >= 0).flatten()
        blk, off = slots[idx] // kc.shape[1], slots[idx] % kc.shape[1]
        assert np.array_equal(okc[blk, off].contiguous().view(torch.uint8).numpy(), rec["k_rows"]), name
        assert np.array_equal(ovc[blk, off].contiguous().view(torch.uint8).numpy(), rec["v_rows"]), name
        if kind != "auto":
            assert np.array_equal(oks[blk, off].numpy(), rec["k_scale_rows"]), name
            assert np.array_equal(ovs[blk, off].numpy(), rec["v_scale_rows"]), name


def test_kv_write_batch_scale_views_alias_the_padding():
    b = workloads.build_kv_write_batch(20, kv_cache_dtype="int8_per_token_head", num_blocks=4)
    ks, vs = b.scale_cache_views()
    assert ks.shape == (4, 16, 2) and ks.dtype == torch.float32
    ks[1, 3, 1] = 2.5
    vs[2, 0, 0] = -1.0
    raw = b.kv_cache.view(torch.uint8)
    assert raw[1, 0, 3, 1, 128:132].view(torch.float32).item() == 2.5
    assert raw[2, 1, 0, 0, 128:132].view(torch.float32).item() == -1.0
    assert (raw[..., :128] == 0x5A).all()  # the data part is untouched


def test_kv_cache_validation_on_cpu():
    b = workloads.build_kv_write_batch(8, num_blocks=2)
    kc, vc = b.caches()
    with pytest.raises(AssertionError, match="unsupported kv_cache_dtype"):
        kv_cache.reshape_and_cache_flash(b.key, b.value, kc, vc, b.slot_mapping, "int4", b.k_scale, b.v_scale)
    with pytest.raises(ValueError, match="flash"):
        kv_cache.reshape_and_cache_flash(b.key, b.value, b.kv_cache, b.kv_cache, b.slot_mapping, "auto", b.k_scale, b.v_scale)
    with pytest.raises(ValueError, match="one entry per token"):
        kv_cache.reshape_and_cache_flash(b.key, b.value, kc, vc, b.slot_mapping[:3], "auto", b.k_scale, b.v_scale)
    with pytest.raises(RuntimeError, match="CUDA"):
        kv_cache.reshape_and_cache_flash(b.key, b.value, kc, vc, b.slot_mapping, "auto", b.k_scale, b.v_scale)
    with pytest.raises(ValueError, match="Per-token-head quantization not supported"):
        kv_cache.reshape_and_cache_flash_per_token_head_quant(b.key, b.value, kc, vc, b.k_scale, b.v_scale, b.slot_mapping)
    with pytest.raises(NotImplementedError):
        kv_cache.rope_and_cache(b.key, b.key, b.value, b.slot_mapping, b.k_scale, True, kc, vc, b.slot_mapping,
                                b.k_scale, b.v_scale, False, False)


def _rn32(f):
    """Round an exact rational to the nearest binary32 (ties to even); normal range only."""
    from fractions import Fraction

    if f == 0:
        return 0.0
    sign = -1 if f < 0 else 1
    a = abs(Fraction(f))
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if a < Fraction(2) ** e:
        e -= 1
    m = a / Fraction(2) ** (e - 23)  # in [2^23, 2^24)
    n = m.numerator // m.denominator
    rem = m - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2):
        n += 1
    return sign * float(Fraction(n) * Fraction(2) ** (e - 23))


def test_fixed_divisor_quotient_is_correctly_rounded():
    """The kernels' x / s for a per-launch scale (the fp8 per-tensor caches): y = RN(1/s),
    q = RN(x y), then twice q <- RN(q + RN_exact(x - s q) y) with exact FMA residuals.
    Checked against the correctly rounded quotient with exact rational arithmetic."""
    from fractions import Fraction

    rng = np.random.default_rng(11)
    bf16 = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    bf16 = bf16[np.isfinite(bf16) & (np.abs(bf16) > 1e-30) & (np.abs(bf16) < 1e30)]
    for s in [0.0125, 0.0089, 0.0173, 0.0121, 1 / 3, 0.37, float(rng.uniform(1e-3, 10))]:
        s = float(np.float32(s))
        fs = Fraction(s)
        y = _rn32(1 / fs)
        fy = Fraction(y)
        xs = np.concatenate([rng.choice(bf16, 1500), (rng.standard_normal(1500) * 50).astype(np.float32)])
        for x in xs.tolist():
            fx = Fraction(x)
            q = _rn32(fx * fy)
            for _ in range(2):
                r = _rn32(fx - fs * Fraction(q))  # exact in binary32 (an FMA residual)
                assert Fraction(r) == fx - fs * Fraction(q)
                q = _rn32(Fraction(q) + Fraction(r) * fy)
            assert q == _rn32(fx / fs), (x, s)
