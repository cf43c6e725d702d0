"""Parity of the sm_100a paged KV-cache writes against the oracle (GPU).

The service's cache update (``do_kv_cache_update``) in every mode it selects
-- plain, fp8 per-tensor, int8 / fp8 per-token-head with the scale inline in
the padded cache row -- and the service's rope-and-cache call
(``do_rope_and_kv_cache_update``: query and key rotated in place, plain or
fp8 caches).  Bar: bit-exact with the oracle (cache bytes, scales, rotated
query and key); padding tokens and untouched slots keep the sentinel bytes.
Where vLLM imports on the GPU box its own Triton kernels are run on the same
inputs as a second opinion: plain caches bit-exact, quantised caches within
one code step on a tiny fraction of elements (its fp32 division is not the
correctly rounded one).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from minicpm_b200 import _lib, kv_cache
from minicpm_b200.workloads import build_kv_write_batch, build_rope_batch
from oracle import kv_write_reference, rope_and_cache_service_reference

pytestmark = pytest.mark.gpu


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().contiguous().view(torch.uint8)


def _run_write(b):
    g = b.to("cuda")
    kc, vc = g.caches()
    if b.kv_cache_dtype.endswith("per_token_head"):
        ks, vs = g.scale_cache_views()
        kv_cache.reshape_and_cache_flash_per_token_head_quant(g.key, g.value, kc, vc, ks, vs, g.slot_mapping)
    else:
        kv_cache.reshape_and_cache_flash(g.key, g.value, kc, vc, g.slot_mapping, b.kv_cache_dtype, g.k_scale, g.v_scale)
    torch.cuda.synchronize()
    return g


def _want(b):
    kc, vc = b.caches()
    ksc = vsc = None
    if b.kv_cache_dtype.endswith("per_token_head"):
        ksc, vsc = (t.clone() for t in b.scale_cache_views())
    return kv_write_reference(
        b.key, b.value, kc, vc, b.slot_mapping, b.kv_cache_dtype, float(b.k_scale), float(b.v_scale), ksc, vsc
    )


def _check_write(b, g):
    okc, ovc, oks, ovs = _want(b)
    kc, vc = g.caches()
    assert torch.equal(_u8(kc), _u8(okc)), "key cache"
    assert torch.equal(_u8(vc), _u8(ovc)), "value cache"
    if oks is not None:
        ks, vs = g.scale_cache_views()
        assert torch.equal(ks.cpu(), oks) and torch.equal(vs.cpu(), ovs), "scales"
    assert torch.equal(g.key.cpu(), b.key) and torch.equal(g.value.cpu(), b.value)
    assert _lib.device_error() == _lib.DEVERR_NONE


@pytest.mark.parametrize(
    "dtype,kh,d,slot_dtype",
    [
        (torch.bfloat16, 2, 128, torch.int64),
        (torch.float16, 4, 64, torch.int32),
        (torch.float32, 1, 256, torch.int64),
        (torch.bfloat16, 8, 128, torch.int32),
    ],
)
def test_plain_cache_write(dtype, kh, d, slot_dtype):
    b = build_kv_write_batch(3001, num_kv_heads=kh, head_dim=d, num_blocks=512, padding_tokens=17, dtype=dtype,
                             slot_dtype=slot_dtype)
    _check_write(b, _run_write(b))


@pytest.mark.parametrize("kind", ["auto", "fp8", "int8_per_token_head"])
def test_padded_token_rows(kind):
    """key / value rows with padding after each token (token stride > heads x head_dim)."""
    b = build_kv_write_batch(777, kv_cache_dtype=kind, num_blocks=64, padding_tokens=5)
    want = _want(b)
    g = b.to("cuda")
    t, kh, d = b.key.shape
    pad_k = torch.zeros(t, kh * d + 64, dtype=b.key.dtype, device="cuda")
    pad_v = torch.zeros_like(pad_k)
    pad_k[:, : kh * d] = g.key.reshape(t, -1)
    pad_v[:, : kh * d] = g.value.reshape(t, -1)
    key = pad_k[:, : kh * d].view(t, kh, d)
    value = pad_v[:, : kh * d].view(t, kh, d)
    assert key.stride(0) == kh * d + 64
    kc, vc = g.caches()
    if kind.endswith("per_token_head"):
        ks, vs = g.scale_cache_views()
        kv_cache.reshape_and_cache_flash_per_token_head_quant(key, value, kc, vc, ks, vs, g.slot_mapping)
    else:
        kv_cache.reshape_and_cache_flash(key, value, kc, vc, g.slot_mapping, kind, g.k_scale, g.v_scale)
    torch.cuda.synchronize()
    assert torch.equal(_u8(kc), _u8(want[0])) and torch.equal(_u8(vc), _u8(want[1]))
    if want[2] is not None:
        ks, vs = g.scale_cache_views()
        assert torch.equal(ks.cpu(), want[2]) and torch.equal(vs.cpu(), want[3])
    assert _lib.device_error() == _lib.DEVERR_NONE


@pytest.mark.parametrize("storage", [torch.float8_e4m3fn, torch.uint8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_per_tensor_cache_write(storage, dtype):
    b = build_kv_write_batch(2048, kv_cache_dtype="fp8", num_blocks=256, padding_tokens=9, dtype=dtype)
    b.kv_cache = b.kv_cache.view(storage)
    g = _run_write(b)
    _check_write(b, g)
    # the boosted rows saturate at +-448 rather than turning into NaN codes
    kc, _ = g.caches()
    codes = _u8(kc)
    assert ((codes & 0x7F) == 0x7E).any() and not ((codes & 0x7F) == 0x7F).any()


@pytest.mark.parametrize("kind", ["fp8", "fp8_per_token_head", "int8_per_token_head"])
def test_quantised_special_values(kind):
    """Signed zeros, bf16 subnormals, tiny, huge and infinite inputs."""
    b = build_kv_write_batch(512, kv_cache_dtype=kind, num_blocks=64)
    specials = torch.tensor([0.0, -0.0, 1e-40, -1e-40, 3e-39, 1e-30, -1e-20, 1e30, -3e38, float("inf"),
                             -float("inf"), 0.0125 * 448.5, -0.0125 * 464.0, 0.0125 * 0.5 ** 10],
                            dtype=torch.float32).to(torch.bfloat16)
    k = b.key.view(-1)
    k[: 37 * specials.numel()] = specials.repeat(37)
    if kind.endswith("per_token_head"):  # one head of all zeros and one of a single signed zero
        b.key[100, 0].zero_()
        b.key[101, 1].zero_()
        b.key[101, 1, 5] = -0.0
        b.key[:20] = torch.where(torch.isinf(b.key[:20].float()), torch.zeros(()), b.key[:20].float()).to(b.key.dtype)
    _check_write(b, _run_write(b))


def test_fp8_e5m2_through_the_c_abi():
    b = build_kv_write_batch(1024, kv_cache_dtype="fp8", num_blocks=128, padding_tokens=4)
    b.kv_cache = b.kv_cache.view(torch.float8_e5m2)
    g = b.to("cuda")
    kc, vc = g.caches()
    p = _lib.KvWriteParams(
        key=g.key.data_ptr(), value=g.value.data_ptr(), key_cache=kc.data_ptr(), value_cache=vc.data_ptr(),
        slot_mapping=g.slot_mapping.data_ptr(), k_scale=g.k_scale.data_ptr(), v_scale=g.v_scale.data_ptr(),
        k_stride_t=g.key.stride(0), k_stride_h=g.key.stride(1), v_stride_t=g.value.stride(0), v_stride_h=g.value.stride(1),
        kc_stride_block=kc.stride(0), kc_stride_tok=kc.stride(1), kc_stride_head=kc.stride(2),
        vc_stride_block=vc.stride(0), vc_stride_tok=vc.stride(1), vc_stride_head=vc.stride(2),
        num_tokens=g.key.shape[0], num_kv_heads=g.key.shape[1], head_dim=g.key.shape[2],
        block_size=kc.shape[1], num_blocks=kc.shape[0], dtype=_lib.DTYPE_BF16, cache_dtype=_lib.DTYPE_FP8_E5M2,
        quant_mode=_lib.KVQ_FP8_PER_TENSOR, slot_dtype=_lib.DTYPE_I64,
    )
    _lib.check(_lib.load().b200_kv_cache_write(ctypes.byref(p), _lib.current_stream(g.key.device)), "e5m2")
    torch.cuda.synchronize()
    from oracle import quantize_per_tensor

    slots = b.slot_mapping.long()
    idx = torch.nonzero(slots >= 0).flatten()
    blk, off = slots[idx] // 16, slots[idx] % 16
    want_k = quantize_per_tensor(b.key[idx], float(b.k_scale), "e5m2")
    want_v = quantize_per_tensor(b.value[idx], float(b.v_scale), "e5m2")
    assert np.array_equal(_u8(kc)[blk.cpu(), off.cpu()].numpy(), want_k)
    assert np.array_equal(_u8(vc)[blk.cpu(), off.cpu()].numpy(), want_v)


@pytest.mark.parametrize("kind", ["int8_per_token_head", "fp8_per_token_head"])
@pytest.mark.parametrize("kh,d", [(2, 128), (4, 64), (1, 256)])
def test_per_token_head_cache_write(kind, kh, d):
    b = build_kv_write_batch(1500, kv_cache_dtype=kind, num_kv_heads=kh, head_dim=d, num_blocks=128, padding_tokens=11)
    _check_write(b, _run_write(b))


def test_out_of_range_slot_is_skipped_and_recorded():
    b = build_kv_write_batch(64, num_blocks=8)
    b.slot_mapping[5] = 8 * 16 + 3  # one past the pool
    g = _run_write(b)
    assert _lib.device_error() == _lib.DEVERR_SLOT_RANGE
    b.slot_mapping[5] = -1  # the oracle's view: that token writes nothing
    okc, ovc, _, _ = _want(b)
    kc, vc = g.caches()
    assert torch.equal(_u8(kc), _u8(okc)) and torch.equal(_u8(vc), _u8(ovc))


def test_empty_batch_is_a_no_op():
    b = build_kv_write_batch(16, num_blocks=2).to("cuda")
    kc, vc = b.caches()
    before = kc.clone()
    kv_cache.reshape_and_cache_flash(b.key[:0], b.value[:0], kc, vc, b.slot_mapping[:0], "auto", b.k_scale, b.v_scale)
    torch.cuda.synchronize()
    assert torch.equal(kc, before)


def _vllm():
    try:
        from vllm.v1.attention.ops import triton_reshape_and_cache_flash as vk
    except Exception as exc:  # pragma: no cover - depends on the image
        pytest.skip(f"vLLM not importable: {exc}")
    return vk


@pytest.mark.parametrize("kind", ["auto", "fp8", "int8_per_token_head", "fp8_per_token_head"])
def test_against_vllm_triton_kernels_on_the_gpu(kind):
    vk = _vllm()
    b = build_kv_write_batch(4096, kv_cache_dtype=kind, num_blocks=512, padding_tokens=13)
    ours = _run_write(b)
    theirs = b.to("cuda")
    kc, vc = theirs.caches()
    try:
        if kind.endswith("per_token_head"):
            ks, vs = theirs.scale_cache_views()
            vk.triton_reshape_and_cache_flash_per_token_head_quant(theirs.key, theirs.value, kc, vc, ks, vs, theirs.slot_mapping)
        else:
            vk.triton_reshape_and_cache_flash(theirs.key, theirs.value, kc, vc, theirs.slot_mapping, kind,
                                              theirs.k_scale, theirs.v_scale)
        torch.cuda.synchronize()
    except Exception as exc:  # pragma: no cover
        pytest.skip(f"vLLM kernel did not run here: {exc}")
    okc, ovc = ours.caches()
    if kind == "auto":
        assert torch.equal(_u8(okc), _u8(kc)) and torch.equal(_u8(ovc), _u8(vc))
        return
    for mine, other in ((okc, kc), (ovc, vc)):
        a, c = _u8(mine).numpy(), _u8(other).numpy()
        if kind.startswith("int8"):
            diff = np.abs(a.view(np.int8).astype(np.int32) - c.view(np.int8).astype(np.int32))
        else:  # adjacent fp8 codes of one sign differ by one in their magnitude bits
            diff = np.where((a & 0x80) == (c & 0x80), np.abs((a & 0x7F).astype(np.int32) - (c & 0x7F)), 255)
            diff = np.where(a == c, 0, diff)
        assert diff.max() <= 1 and (diff > 0).mean() < 1e-3, (kind, int(diff.max()), float((diff > 0).mean()))
    if kind.endswith("per_token_head"):
        ks_o, vs_o = ours.scale_cache_views()
        ks_t, vs_t = theirs.scale_cache_views()
        slots = b.slot_mapping.long()
        slots = slots[slots >= 0]
        blk, off = slots // 16, slots % 16
        for x, y in ((ks_o, ks_t), (vs_o, vs_t)):
            x, y = x.cpu()[blk, off], y.cpu()[blk, off]
            assert ((x - y).abs() / y.abs()).max().item() <= 2.5e-7


# --- the service's rope-and-cache call -------------------------------------------------


def _service_run(b, apply_scale, storage=None):
    g = b.to("cuda")
    kc, vc = g.key_cache, g.value_cache
    ks = torch.tensor([0.0173], device="cuda")
    vs = torch.tensor([0.0121], device="cuda")
    if apply_scale:
        kc = torch.full(kc.shape, 0x5A, dtype=torch.uint8, device="cuda").view(storage)
        vc = torch.full(vc.shape, 0x5A, dtype=torch.uint8, device="cuda").view(storage)
    kc0, vc0 = kc.clone(), vc.clone()
    kv_cache.rope_and_cache(g.query, g.key, g.value, g.positions, g.cos_sin_cache, g.is_neox, kc, vc, g.slot_mapping,
                            ks, vs, True, apply_scale)
    torch.cuda.synchronize()
    want = rope_and_cache_service_reference(
        b.query, b.key, b.value, b.positions, b.cos_sin_cache, b.is_neox, kc0.cpu(), vc0.cpu(), b.slot_mapping,
        float(ks), float(vs), apply_scale,
    )
    return g, kc, vc, want


@pytest.mark.parametrize("is_neox", [True, False])
@pytest.mark.parametrize("rd", [64, 128])
@pytest.mark.parametrize("fp8", [False, True])
def test_service_rope_and_cache(is_neox, rd, fp8):
    b = build_rope_batch(4096, rotary_dim=rd, is_neox=is_neox, num_blocks=512)
    b.slot_mapping[-7:] = -1
    g, kc, vc, (q_want, k_want, kc_want, vc_want) = _service_run(b, fp8, torch.float8_e4m3fn)
    assert torch.equal(_u8(g.query), _u8(q_want)), "query rotated in place"
    assert torch.equal(_u8(g.key), _u8(k_want)), "key rotated in place (k_out = key), every token"
    assert torch.equal(_u8(kc), _u8(kc_want)), "key cache"
    assert torch.equal(_u8(vc), _u8(vc_want)), "value cache"
    assert torch.equal(g.value.cpu(), b.value)
    assert _lib.device_error() == _lib.DEVERR_NONE


def test_service_rope_and_cache_uint8_storage():
    b = build_rope_batch(1024, rotary_dim=128, is_neox=True, num_blocks=128)
    g, kc, vc, (_, _, kc_want, vc_want) = _service_run(b, True, torch.uint8)
    assert torch.equal(_u8(kc), _u8(kc_want)) and torch.equal(_u8(vc), _u8(vc_want))
