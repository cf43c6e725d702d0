"""The service shim's host logic on CPU: routing, the descale guard, metadata, backend contract.

Routes are observed by replacing the two targets (vLLM's ``unified_attention``
and the sm_100a ``unified_attention_optimized``) with recorders; nothing here
launches a kernel.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from minicpm_b200 import service


@pytest.fixture
def routes(monkeypatch):
    calls = []
    monkeypatch.setattr(service, "_vllm_unified_attention", lambda: (lambda **kw: calls.append(("vllm", kw))))
    monkeypatch.setattr(service, "unified_attention_optimized", lambda **kw: calls.append(("b200", kw)))
    for name in ("ILUVATAR_USE_OPTIMIZED", "ILUVATAR_SPLIT_KV", "ILUVATAR_SPLIT_KV_DECODE", "ILUVATAR_NUM_SPLITS"):
        monkeypatch.delenv(name, raising=False)
    return calls


def _qk(hq=16, hkv=2, d=128, dtype=torch.bfloat16):
    """Shape-only tensors (meta device: no storage) for the route's shape check."""
    q = torch.empty(64, hq, d, dtype=dtype, device="meta")
    k = torch.empty(8, 16, hkv, d, dtype=dtype, device="meta")
    return q, k


def _kwargs(**over):
    q, k = _qk()
    kw = dict(q=q, k=k, v=k, out=q, cu_seqlens_q=None, max_seqlen_q=64, seqused_k=None, max_seqlen_k=100,
              softmax_scale=0.1, causal=True, block_table=None, alibi_slopes=None, window_size=(-1, -1), softcap=0.0,
              q_descale=None, k_descale=None, v_descale=None, sinks=None, kv_quant_mode=service.KVQuantMode.NONE,
              use_td=False)
    kw.update(over)
    return kw


@pytest.mark.parametrize("flags", ["1", "true", "YES"])
def test_enabled_prefill_goes_to_b200(routes, monkeypatch, flags):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", flags)
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", flags)
    service._run_unified_attention(**_kwargs())
    assert routes[-1][0] == "b200"
    assert routes[-1][1]["num_splits_override"] is None  # automatic split count


def test_num_splits_env_is_forwarded(routes, monkeypatch):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    monkeypatch.setenv("ILUVATAR_NUM_SPLITS", "8")
    service._run_unified_attention(**_kwargs())
    assert routes[-1][1]["num_splits_override"] == 8


@pytest.mark.parametrize(
    "over",
    [
        dict(kv_quant_mode=service.KVQuantMode.FP8_PER_TENSOR),
        dict(alibi_slopes=torch.ones(4)),
        dict(sinks=torch.ones(4)),
        dict(softcap=30.0),
        dict(window_size=(127, 0)),
        dict(q_descale=torch.ones(1)),
        dict(k_descale=torch.ones(1)),
        dict(v_descale=torch.ones(1)),
        dict(use_td=True),
        dict(causal=False),
        dict(max_seqlen_q=1),
        dict(max_seqlen_q=0),
    ],
)
def test_unsupported_features_and_decode_stay_on_vllm(routes, monkeypatch, over):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    service._run_unified_attention(**_kwargs(**over))
    assert routes[-1][0] == "vllm"


@pytest.mark.parametrize(
    "shape,route",
    [
        (dict(d=256), "b200"),  # head_dim 256: the kernel's wide variant
        (dict(d=96), "vllm"),  # a head size the sm_100a kernel does not run
        (dict(hq=12, hkv=2), "b200"),  # GQA 6:1 (128 rows hold 21 positions x 6 heads)
        (dict(hq=24, hkv=2), "b200"),  # GQA 12:1
        (dict(hq=256, hkv=1), "vllm"),  # more than 128 query heads per KV head
        (dict(dtype=torch.float32), "vllm"),
        (dict(d=64), "b200"),
    ],
)
def test_shapes_the_kernel_does_not_run_go_to_vllm(routes, monkeypatch, shape, route):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    q, k = _qk(**shape)
    service._run_unified_attention(**_kwargs(q=q, k=k, v=k, out=q))
    assert routes[-1][0] == route


def test_decode_flag_routes_decode_to_b200(routes, monkeypatch):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV_DECODE", "1")
    service._run_unified_attention(**_kwargs(max_seqlen_q=1))
    assert routes[-1][0] == "b200"


@pytest.mark.parametrize("env", [{}, {"ILUVATAR_USE_OPTIMIZED": "1"}, {"ILUVATAR_SPLIT_KV": "1"}])
def test_both_flags_are_required(routes, monkeypatch, env):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    service._run_unified_attention(**_kwargs())
    assert routes[-1][0] == "vllm"


def test_b200_failures_propagate(monkeypatch):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")

    def boom(**kw):
        raise RuntimeError("kernel failed")

    monkeypatch.setattr(service, "unified_attention_optimized", boom)
    monkeypatch.setattr(service, "_vllm_unified_attention", lambda: pytest.fail("silent fallback to vLLM"))
    with pytest.raises(RuntimeError, match="kernel failed"):
        service._run_unified_attention(**_kwargs())


def _metadata(max_query_len=4, num_tokens=8, seqs=2):
    b = service.IluvatarAttentionMetadataBuilder(16, 2, 128, torch.device("cpu"))
    common = SimpleNamespace(
        num_reqs=seqs, num_actual_tokens=num_tokens, max_query_len=max_query_len, max_seq_len=100,
        query_start_loc=torch.tensor([0, 4, 8], dtype=torch.int32), seq_lens=torch.tensor([50, 100], dtype=torch.int32),
        block_table_tensor=torch.zeros(2, 8, dtype=torch.int32), slot_mapping=torch.arange(num_tokens), causal=True,
    )
    return b, b.build(0, common)


def _impl(kv_cache_dtype="auto", **kw):
    return service.IluvatarAttentionImpl(16, 128, 0.088, 2, None, None, kv_cache_dtype, **kw)


def _layer():
    return SimpleNamespace(_k_scale=torch.tensor(1.0), _v_scale=torch.tensor(1.0), _q_scale=torch.tensor(1.0))


def test_forward_passes_no_descale_for_unquantised_caches(routes, monkeypatch):
    # The reference passed layer scales here, which the route treats as
    # unsupported: the optimized path was unreachable in the service.
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    _, meta = _metadata()
    kv_cache = torch.zeros(8, 2, 16, 2, 128, dtype=torch.bfloat16)
    q = torch.zeros(8, 16, 128, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    _impl().forward(_layer(), q, q, q, kv_cache, meta, out)
    name, kw = routes[-1]
    assert name == "b200"
    assert kw["k"].shape == (8, 16, 2, 128)  # kv_cache.unbind(1)


def test_forward_fp8_cache_passes_descales_to_the_dequantising_path(routes, monkeypatch):
    """An fp8 per-tensor cache with its descales takes the sm_100a path (its
    pages are dequantised first); the reference sent it to vLLM."""
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    _, meta = _metadata()
    kv_cache = torch.zeros(8, 2, 16, 2, 128, dtype=torch.uint8)
    q = torch.zeros(8, 16, 128, dtype=torch.bfloat16)
    _impl("fp8").forward(_layer(), q, q, q, kv_cache, meta, torch.empty_like(q))
    name, kw = routes[-1]
    assert name == "b200"
    assert kw["k_descale"].shape == (2, 2) and kw["k"].dtype == torch.float8_e4m3fn
    assert kw["kv_quant_mode"] == service.KVQuantMode.FP8_PER_TENSOR


def test_forward_per_token_head_cache_takes_the_dequantising_path(routes, monkeypatch):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    _, meta = _metadata()
    kv_cache = torch.zeros(8, 2, 16, 2, 132, dtype=torch.int8)
    q = torch.zeros(8, 16, 128, dtype=torch.bfloat16)
    _impl("int8_per_token_head").forward(_layer(), q, q, q, kv_cache, meta, torch.empty_like(q))
    name, kw = routes[-1]
    assert name == "b200" and kw["kv_quant_mode"] == service.KVQuantMode.INT8_PER_TOKEN_HEAD
    assert kw["k_scale_cache"].shape == (8, 16, 2) and kw["k_descale"] is None


@pytest.mark.parametrize("over", [
    dict(kv_quant_mode=service.KVQuantMode.NVFP4),
    dict(kv_quant_mode=service.KVQuantMode.INT8_PER_TOKEN_HEAD),  # no scale caches
    dict(kv_quant_mode=service.KVQuantMode.FP8_PER_TENSOR, k_descale=torch.ones(1)),  # no v_descale
])
def test_quantised_caches_without_what_they_need_stay_on_vllm(routes, monkeypatch, over):
    monkeypatch.setenv("ILUVATAR_USE_OPTIMIZED", "1")
    monkeypatch.setenv("ILUVATAR_SPLIT_KV", "1")
    q, _ = _qk()
    k = torch.empty(8, 16, 2, 128, dtype=torch.int8, device="meta")
    service._run_unified_attention(**_kwargs(q=q, k=k, v=k, out=q, **over))
    assert routes[-1][0] == "vllm"


def test_forward_per_token_head_cache_sets_up_inline_scales(routes):
    _, meta = _metadata()
    kv_cache = torch.zeros(8, 2, 16, 2, 132, dtype=torch.int8)
    q = torch.zeros(8, 16, 128, dtype=torch.bfloat16)
    impl = _impl("int8_per_token_head")
    impl.forward(_layer(), q, q, q, kv_cache, meta, torch.empty_like(q))
    name, kw = routes[-1]
    assert name == "vllm" and kw["k_descale"] is None
    assert kw["k_scale_cache"].shape == (8, 16, 2)
    # the scale views alias the 4 bytes after head_size and start at 1.0
    assert kv_cache.view(torch.uint8)[3, 1, 5, 1, 128:132].view(torch.float32).item() == 1.0
    kw["v_scale_cache"][3, 5, 1] = 2.0
    assert kv_cache.view(torch.uint8)[3, 1, 5, 1, 128:132].view(torch.float32).item() == 2.0


def test_forward_profiling_run_and_guards():
    impl = _impl()
    out = torch.ones(4, 16, 128)
    assert impl.forward(_layer(), out, out, out, out, None, out).abs().sum() == 0
    with pytest.raises(NotImplementedError):
        impl.forward(_layer(), out, out, out, out, None, out, output_block_scale=torch.ones(1))
    _, meta = _metadata()
    meta.use_cascade = True
    with pytest.raises(AssertionError):
        impl.forward(_layer(), out, out, out, out, meta, out)


def test_metadata_builder_and_backend_contract():
    b, meta = _metadata()
    assert meta.seq_threshold_3D == 64 and meta.num_par_softmax_segments == 16
    assert meta.softmax_segm_output.shape == (64, 16, 16, 128)
    assert meta.use_cascade is False and meta.max_query_len == 4
    gb = service.IluvatarAttentionMetadataBuilder(16, 2, 128, torch.device("cpu"), cudagraph_capture_sizes=[1, 2, 48, 80])
    assert gb.seq_threshold_3D == 48
    be = service.IluvatarAttentionBackend
    assert be.get_name() == "TRITON_ATTN" and be.get_impl_cls() is service.IluvatarAttentionImpl
    assert be.get_kv_cache_shape(10, 16, 2, 128) == (10, 2, 16, 2, 128)
    assert be.get_kv_cache_shape(10, 16, 2, 128, "fp8_per_token_head") == (10, 2, 16, 2, 132)
    with pytest.raises(ValueError):
        be.get_kv_cache_shape(10, 24, 2, 128)
    assert be.supports_block_size(32) and not be.supports_block_size(24)
    assert be.get_kv_cache_stride_order() == (0, 1, 2, 3, 4)
    assert service.get_kv_quant_mode("fp8_e5m2") == service.KVQuantMode.FP8_PER_TENSOR
    assert not _impl("int8_per_token_head").fused_rope_kvcache_supported() and _impl("fp8").fused_rope_kvcache_supported()
