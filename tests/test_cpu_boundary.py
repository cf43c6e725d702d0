"""Host-side boundary tests (no GPU): the C-ABI library, validation, routing.

* the built library loads and exports every function ``include/*.h`` declares;
* the operators raise the reference's ``ValueError`` messages
  (kernels/triton_split_kv_paged.py:249-281, kernels/triton_rope_kv_cache.py:219-260)
  before touching a device;
* the dispatcher routes as kernels/attention.py:99-167 does;
* the split-count resolution order of
  kernels/triton_unified_attention_optimized.py:216-218 (plus automatic 0).
"""

from __future__ import annotations

import re
from pathlib import Path

import pytest
import torch

import minicpm_b200
from minicpm_b200 import _lib, attention, fused_rope_and_cache, paged_split_kv_attention
from minicpm_b200.unified_attention_optimized import resolve_num_splits, unified_attention_optimized

ROOT = Path(__file__).resolve().parent.parent


def _declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(b200_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert set(_lib.EXPORTED_SYMBOLS) <= declared
    assert lib.b200_abi_version() == _lib.ABI_VERSION == 2


def test_host_only_entry_points():
    lib = _lib.load()
    # No GPU here: the SM count falls back to 148.
    assert lib.b200_choose_num_splits(32768, 64, 16, 2, 4096) == 1
    assert lib.b200_choose_num_splits(16, 1, 16, 2, 16384) > 1
    assert lib.b200_choose_num_splits(16, 1, 16, 2, 300) == 1
    small = lib.b200_attn_workspace_bytes(484, 4, 16, 2, 128, 1, 2302, _lib.DTYPE_BF16)
    split = lib.b200_attn_workspace_bytes(484, 4, 16, 2, 128, 4, 2302, _lib.DTYPE_BF16)
    assert split >= small + 4 * 484 * 16 * (128 * 2 + 8)


def test_invalid_params_return_status_not_crash():
    lib = _lib.load()
    import ctypes

    p = _lib.AttnParams(dtype=_lib.DTYPE_F32, num_q_heads=16, num_kv_heads=2, head_dim=128, block_size=16)
    assert lib.b200_paged_attn_fwd(ctypes.byref(p), None) == _lib.B200_ERR_UNSUPPORTED
    p = _lib.AttnParams(dtype=_lib.DTYPE_BF16, num_q_heads=16, num_kv_heads=3, head_dim=128, block_size=16)
    assert lib.b200_paged_attn_fwd(ctypes.byref(p), None) == _lib.B200_ERR_INVALID
    assert "head shape" in lib.b200_last_error().decode()
    r = _lib.RopeParams(dtype=_lib.DTYPE_BF16, position_dtype=_lib.DTYPE_I32, slot_dtype=_lib.DTYPE_I32,
                        cos_sin_dtype=_lib.DTYPE_BF16, rotary_dim=3, head_dim=128, num_q_heads=16, num_kv_heads=2,
                        block_size=16)
    assert lib.b200_rope_kv_write(ctypes.byref(r), None) == _lib.B200_ERR_INVALID
    c = _lib.CombineParams(num_splits=17, num_heads=16, head_dim=128)
    assert lib.b200_split_combine(ctypes.byref(c), None) == _lib.B200_ERR_INVALID
    if not torch.cuda.is_available():  # the launch itself fails with a status, not a crash
        assert lib.b200_wait_selftest(None) == _lib.B200_ERR_CUDA


def _attn_args(**over):
    q = torch.zeros(8, 16, 128, dtype=torch.bfloat16)
    k = torch.zeros(4, 16, 2, 128, dtype=torch.bfloat16)
    args = dict(
        q=q, k=k, v=k.clone(), out=torch.empty_like(q), block_table=torch.zeros(1, 4, dtype=torch.int32),
        seqused_k=torch.tensor([8], dtype=torch.int32), cu_seqlens_q=torch.tensor([0, 8], dtype=torch.int32),
        max_seqlen_q=8, max_seqlen_k=8, softmax_scale=0.1,
    )
    args.update(over)
    return args


@pytest.mark.parametrize(
    "over,msg",
    [
        (dict(q=torch.zeros(8, 16 * 128)), "expected q=[T,H,D]"),
        (dict(out=torch.empty(7, 16, 128)), "out must match q"),
        (dict(num_splits=3), "num_splits must be one of 2, 4, 8, 16"),
        (dict(num_splits=32), "num_splits must be one of 2, 4, 8, 16"),
        (dict(block_table=torch.zeros(1, 4)), "block_table must contain integer physical block ids"),
        (dict(cu_seqlens_q=torch.tensor([[0, 8]], dtype=torch.int32)), "one-dimensional"),
        (dict(cu_seqlens_q=torch.tensor([0, 4, 8], dtype=torch.int32)), "one entry per request plus one"),
        (dict(block_table=torch.zeros(2, 4, dtype=torch.int32)), "same request count"),
        (dict(q=torch.zeros(8, 16, 96), out=torch.zeros(8, 16, 96)), "unsupported head shape"),
        (dict(block_m=24), "unsupported head shape"),
        (dict(k=torch.zeros(4, 8, 2, 128), v=torch.zeros(4, 8, 2, 128)), "unsupported head shape"),
    ],
)
def test_attention_validation_messages(over, msg):
    with pytest.raises(ValueError, match=re.escape(msg)):
        paged_split_kv_attention(**_attn_args(**over))


def test_attention_zero_lengths_zero_out_on_cpu_without_kernel():
    args = _attn_args(max_seqlen_q=0)
    args["out"].fill_(5)
    assert paged_split_kv_attention(**args).abs().max().item() == 0


def test_attention_cpu_tensors_are_refused_not_computed():
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        paged_split_kv_attention(**_attn_args())


def test_non_causal_is_rejected():
    with pytest.raises(ValueError, match="causal attention only"):
        unified_attention_optimized(**_attn_args(), causal=False)


def _rope_args(**over):
    args = dict(
        query=torch.zeros(4, 16, 128, dtype=torch.bfloat16), key=torch.zeros(4, 2, 128, dtype=torch.bfloat16),
        value=torch.zeros(4, 2, 128, dtype=torch.bfloat16), positions=torch.zeros(4, dtype=torch.int32),
        cos_sin_cache=torch.zeros(16, 128, dtype=torch.bfloat16), is_neox=True,
        key_cache=torch.zeros(2, 16, 2, 128, dtype=torch.bfloat16), value_cache=torch.zeros(2, 16, 2, 128, dtype=torch.bfloat16),
        slot_mapping=torch.zeros(4, dtype=torch.int32),
    )
    args.update(over)
    return args


@pytest.mark.parametrize(
    "over,msg",
    [
        (dict(query=torch.zeros(4, 2048, dtype=torch.bfloat16)), "query/key/value must have shape"),
        (dict(key_cache=torch.zeros(2, 16, 256, dtype=torch.bfloat16)), "only NHD paged KV cache"),
        (dict(key=torch.zeros(4, 2, 128, dtype=torch.float16)), "must share a dtype"),
        (dict(value_cache=torch.zeros(2, 32, 2, 128, dtype=torch.bfloat16)), "cache shapes must match"),
        (dict(value_cache=torch.zeros(2, 2, 16, 128, dtype=torch.bfloat16).transpose(1, 2)), "cache strides must match"),
        (dict(query=torch.zeros(4, 16, 128), key=torch.zeros(4, 2, 128), value=torch.zeros(4, 2, 128)), "only unquantized BF16/FP16"),
        (dict(positions=torch.zeros(4)), "integer indices"),
        (dict(slot_mapping=torch.zeros(3, dtype=torch.int32)), "one entry per token"),
        (dict(cos_sin_cache=torch.zeros(16, 127, dtype=torch.bfloat16)), "cos_sin_cache must be"),
        (dict(rotary_dim=64), "unsupported RoPE/cache shape"),
        (dict(key_cache=torch.zeros(2, 8, 2, 128, dtype=torch.bfloat16), value_cache=torch.zeros(2, 8, 2, 128, dtype=torch.bfloat16)), "unsupported RoPE/cache shape"),
    ],
)
def test_rope_validation_messages(over, msg):
    with pytest.raises(ValueError, match=re.escape(msg)):
        fused_rope_and_cache(**_rope_args(**over))


def test_rope_cpu_tensors_are_refused_not_computed():
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fused_rope_and_cache(**_rope_args())


def test_split_resolution_order(monkeypatch):
    monkeypatch.delenv("ILUVATAR_NUM_SPLITS", raising=False)
    monkeypatch.delenv("VLLM_ILUVATAR_ATTN_SPLIT_KV_SEGMENTS", raising=False)
    assert resolve_num_splits(None) == 0  # automatic
    monkeypatch.setenv("VLLM_ILUVATAR_ATTN_SPLIT_KV_SEGMENTS", "8")
    assert resolve_num_splits(None) == 8
    monkeypatch.setenv("ILUVATAR_NUM_SPLITS", "2")
    assert resolve_num_splits(None) == 2
    assert resolve_num_splits(16) == 16


class _Recorder:
    def __init__(self):
        self.calls = []

    def __call__(self, **kw):
        self.calls.append(kw)
        return kw["out"]


def _dispatch_args(**over):
    a = _attn_args()
    args = dict(q=a["q"], k=a["k"], v=a["v"], out=a["out"], cu_seqlens_q=a["cu_seqlens_q"], max_seqlen_q=8,
                seqused_k=a["seqused_k"], max_seqlen_k=8, softmax_scale=0.1, block_table=a["block_table"])
    args.update(over)
    return args


@pytest.fixture
def routes(monkeypatch):
    baseline, optimized = _Recorder(), _Recorder()
    monkeypatch.setattr(attention, "_vllm_unified_attention", lambda: baseline)
    monkeypatch.setattr(attention, "unified_attention_optimized", optimized)
    return baseline, optimized


def test_dispatcher_flags_off_go_to_vllm(routes, monkeypatch):
    baseline, optimized = routes
    monkeypatch.delenv("ILUVATAR_USE_OPTIMIZED", raising=False)
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    minicpm_b200.iluvatar_attention(**_dispatch_args())
    assert len(baseline.calls) == 1 and not optimized.calls


@pytest.mark.parametrize(
    "over",
    [dict(max_seqlen_q=1), dict(softcap=30.0), dict(kv_quant_mode=1), dict(alibi_slopes=torch.zeros(16)),
     dict(window_size=(128, 0)), dict(q_descale=torch.ones(1)), dict(sinks=torch.zeros(16)), dict(use_td=True)],
)
def test_dispatcher_unsupported_features_go_to_vllm(routes, monkeypatch, over):
    baseline, optimized = routes
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    minicpm_b200.iluvatar_attention(**_dispatch_args(**over))
    assert len(baseline.calls) == 1 and not optimized.calls


@pytest.mark.parametrize("hq,hkv,d,dtype,optimized_route", [
    (16, 2, 256, torch.bfloat16, True), (16, 2, 96, torch.bfloat16, False), (16, 2, 128, torch.float32, False),
    (256, 1, 128, torch.bfloat16, False),
    (12, 2, 128, torch.bfloat16, True), (16, 2, 64, torch.float16, True)])
def test_dispatcher_routes_shapes_the_kernel_does_not_run_to_vllm(routes, monkeypatch, hq, hkv, d, dtype,
                                                                  optimized_route):
    baseline, optimized = routes
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    q = torch.empty(8, hq, d, dtype=dtype, device="meta")
    cache = torch.empty(4, 2, 16, hkv, d, dtype=dtype, device="meta")
    minicpm_b200.iluvatar_attention(**_dispatch_args(q=q, k=cache, v=cache, out=q))
    assert (len(optimized.calls), len(baseline.calls)) == ((1, 0) if optimized_route else (0, 1))


def test_dispatcher_quantised_caches_take_the_dequantising_route(routes, monkeypatch):
    """fp8 per-tensor with descales, int8 per-token-head with scale caches:
    the optimized route, with the scales forwarded; without them: vLLM."""
    baseline, optimized = routes
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    fp8 = torch.empty(4, 2, 16, 2, 128, dtype=torch.float8_e4m3fn, device="meta")
    minicpm_b200.iluvatar_attention(**_dispatch_args(k=fp8, v=fp8, kv_quant_mode=1, k_descale=torch.ones(1, 2),
                                                     v_descale=torch.ones(1, 2)))
    assert len(optimized.calls) == 1 and optimized.calls[0]["kv_quant_mode"] == 1
    assert optimized.calls[0]["k_descale"] is not None
    i8 = torch.empty(4, 2, 16, 2, 132, dtype=torch.int8, device="meta")
    sc = torch.ones(4, 16, 2)
    minicpm_b200.iluvatar_attention(**_dispatch_args(k=i8, v=i8, kv_quant_mode=2, k_scale_cache=sc, v_scale_cache=sc))
    assert len(optimized.calls) == 2 and optimized.calls[1]["k_scale_cache"] is sc
    minicpm_b200.iluvatar_attention(**_dispatch_args(k=i8, v=i8, kv_quant_mode=2))
    assert len(baseline.calls) == 1


def test_dispatcher_optimized_route_and_5d_unbind(routes, monkeypatch):
    baseline, optimized = routes
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    monkeypatch.setenv("ILUVATAR_NUM_SPLITS", "8")
    cache = torch.zeros(4, 2, 16, 2, 128, dtype=torch.bfloat16)
    minicpm_b200.iluvatar_attention(**_dispatch_args(k=cache, v=cache, k_descale=torch.ones(1)))
    assert not baseline.calls and len(optimized.calls) == 1
    kw = optimized.calls[0]
    assert kw["k"].shape == (4, 16, 2, 128) and kw["k"].data_ptr() == cache[:, 0].data_ptr()
    assert kw["v"].data_ptr() == cache[:, 1].data_ptr()
    assert kw["num_splits_override"] == 8 and kw["block_m_override"] == 64


def test_dispatcher_without_vllm_raises(monkeypatch):
    monkeypatch.setattr(attention, "_vllm_unified_attention", lambda: None)
    monkeypatch.delenv("ILUVATAR_USE_OPTIMIZED", raising=False)
    with pytest.raises(RuntimeError, match="vLLM baseline unavailable"):
        minicpm_b200.iluvatar_attention(**_dispatch_args())
