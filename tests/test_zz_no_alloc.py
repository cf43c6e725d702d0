"""The allocation-free attention entry point, ``b200_paged_attn_fwd_noalloc``.

It exists for callers that cannot allocate device memory when they call in:
an engine that reserved nearly all HBM for its KV-cache pages at start-up, a
host runtime in another language that reaches the library only through the
C ABI and has no device allocator, or a latency-critical path where
cudaMalloc/cudaFree would synchronise the device.  It runs the same kernels
as ``b200_paged_attn_fwd`` with the scratch in a fixed-size device array
inside the library instead of a caller-owned workspace.

The GPU tests call it through the C ABI (ctypes, no torch in between) and
check its output against the existing entry point's on calls in a row that
alternate prefill and decode batches, with and without a split KV axis and
with the automatic split count (the split case keeps the partial outputs in
the static array).  This file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import ATOL_MAX, ATOL_MEAN, errors
from minicpm_b200 import _lib, paged_split_kv_attention
from minicpm_b200.workloads import build_attention_batch, correctness_batch


def _params(b, out, num_splits):
    return _lib.AttnParams(
        q=b.q.data_ptr(), k=b.kv_cache[:, 0].data_ptr(), v=b.kv_cache[:, 1].data_ptr(), out=out.data_ptr(),
        block_table=b.block_table.data_ptr(), cu_seqlens_q=b.cu_seqlens_q.data_ptr(), seqused_k=b.seqused_k.data_ptr(),
        q_stride_t=b.q.stride(0), q_stride_h=b.q.stride(1),
        k_stride_block=b.kv_cache.stride(0), k_stride_tok=b.kv_cache.stride(2), k_stride_head=b.kv_cache.stride(3),
        v_stride_block=b.kv_cache.stride(0), v_stride_tok=b.kv_cache.stride(2), v_stride_head=b.kv_cache.stride(3),
        out_stride_t=out.stride(0), out_stride_h=out.stride(1),
        block_table_stride=b.block_table.stride(0), block_table_cols=b.block_table.shape[1],
        block_table_dtype=_lib.DTYPE_I32, seqlen_dtype=_lib.DTYPE_I32, dtype=_lib.DTYPE_BF16,
        num_seqs=len(b.query_lens), total_q=b.q.shape[0], num_q_heads=b.q.shape[1], num_kv_heads=b.kv_cache.shape[3],
        head_dim=b.q.shape[2], block_size=b.kv_cache.shape[2], num_blocks=b.kv_cache.shape[0],
        max_seqlen_q=b.max_seqlen_q, max_seqlen_k=b.max_seqlen_k, num_splits=num_splits,
        softmax_scale=b.softmax_scale, workspace=None, workspace_bytes=0,
    )


def _noalloc(b, num_splits):
    lib = _lib.load()
    out = torch.full_like(b.q, float("nan"))
    p = _params(b, out, num_splits)
    status = lib.b200_paged_attn_fwd_noalloc(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == _lib.B200_OK, lib.b200_last_error().decode()
    torch.cuda.synchronize()
    return out


def _existing(b, num_splits):
    out = torch.empty_like(b.q)
    paged_split_kv_attention(b.q, b.kv_cache[:, 0], b.kv_cache[:, 1], out, b.block_table, b.seqused_k,
                             b.cu_seqlens_q, b.max_seqlen_q, b.max_seqlen_k, b.softmax_scale, num_splits=num_splits)
    torch.cuda.synchronize()
    return out


def _assert_matches(got, want, tag):
    assert torch.isfinite(got.float()).all(), tag
    mx, mn = errors(got.cpu(), want.cpu())
    assert mx <= ATOL_MAX and mn <= ATOL_MEAN, f"{tag}: max={mx} mean={mn}"


@pytest.mark.gpu
@pytest.mark.parametrize("num_splits", [1, 4, 0])
def test_noalloc_matches_existing_entry_point_two_calls(num_splits):
    """Prefill and decode batches interleaved, so each call reads scratch that
    a call of the other layout wrote (the decode kernel keeps item offsets, an
    order list and fp32 partials there; the prefill kernel its work list and,
    when split, the partial outputs and m / l)."""
    _lib.load().b200_paged_attn_fwd_noalloc.argtypes = [ctypes.POINTER(_lib.AttnParams), ctypes.c_void_p]
    first = correctness_batch().to("cuda")
    second = build_attention_batch([3, 200, 1], [40, 900, 77], seed=41).to("cuda")
    # One query token per sequence, 8 query heads per KV head: the decode kernel.
    decode = build_attention_batch([1] * 9, [5, 700, 2049, 16, 4096, 1, 300, 129, 1500], seed=43).to("cuda")
    decode2 = build_attention_batch([1] * 3, [8000, 33, 257], seed=44).to("cuda")
    calls = [("prefill 1", first), ("decode 1", decode), ("prefill 2", second), ("decode 2", decode2),
             ("prefill 1 again", first), ("decode 1 again", decode)]
    want = {tag: _existing(b, num_splits) for tag, b in calls}
    # Calls in a row on different batches: each must match the workspace
    # entry point despite the shared scratch.
    for tag, b in calls:
        _assert_matches(_noalloc(b, num_splits), want[tag], f"{tag} S={num_splits}")
    assert _lib.device_error() == _lib.DEVERR_NONE


def test_noalloc_rejects_sizes_beyond_the_static_scratch():
    lib = _lib.load()
    lib.b200_paged_attn_fwd_noalloc.argtypes = [ctypes.POINTER(_lib.AttnParams), ctypes.c_void_p]
    p = _lib.AttnParams(dtype=_lib.DTYPE_BF16, num_seqs=64, total_q=131072, num_q_heads=16, num_kv_heads=2,
                        head_dim=128, block_size=16, num_blocks=1, block_table_cols=1, num_splits=16,
                        max_seqlen_k=16384, max_seqlen_q=2048)
    assert lib.b200_paged_attn_fwd_noalloc(ctypes.byref(p), None) == _lib.B200_ERR_INVALID
    assert "static scratch" in lib.b200_last_error().decode()
