"""fp32 CPU restatement of the reference's paged causal attention semantics.

TEST INFRASTRUCTURE ONLY (the checker and the CPU baseline; never shipped).

Reference files followed (paths inside the reference project):

* ``tests/test_paged_split_kv.py:19-50`` and ``tests/attention_harness.py:118-145``
  -- the fp32 paged-SDPA reference: gather the row's pages from the block
  table, truncate to the sequence length, repeat KV heads for GQA, einsum in
  fp32, causal mask ``k <= prefix + i``, softmax, einsum, cast.
* ``kernels/triton_split_kv_paged.py:63-155`` -- Split-KV partial semantics:
  ``split_size = ceil(L / S)``, split ``s`` covers keys
  ``[s * size, min((s + 1) * size, L))``; the query's absolute position is
  ``L - q_len + i``; a row with no valid key in a split keeps ``m = -inf``,
  ``l = 0`` and stores ``O = acc / max(l, 1e-20) = 0``.
* ``kernels/triton_split_kv_paged.py:197-228`` -- the cross-split reduce:
  ``m* = max_s m_s``; ``w_s = exp(m_s - m*) * l_s`` for ``l_s > 0`` else 0;
  ``out = sum_s w_s O_s / max(sum_s w_s, 1e-20)``.

One deliberate difference from ``tests/test_paged_split_kv.py:47``: a query
row that sees no key at all (only possible when ``seqused_k < q_len``) is 0
here, as the kernels produce, instead of the NaN that ``softmax`` over an
all ``-inf`` row gives.
"""

from __future__ import annotations

import math
from typing import Sequence

import torch


def causal_flops(query_lens: Sequence[int], kv_lens: Sequence[int], num_q_heads: int, head_dim: int) -> int:
    """Causal FLOP count of ``tests/attention_harness.py:381-385``.

    ``4 * sum_i (q_i * p_i + q_i (q_i + 1) / 2) * H * D`` with ``p_i = L_i - q_i``
    the prior context of sequence ``i``.
    """
    pairs = 0
    for q, L in zip(query_lens, kv_lens):
        p = L - q
        pairs += q * p + q * (q + 1) // 2
    return 4 * pairs * num_q_heads * head_dim


def _gather_sequence_kv(cache: torch.Tensor, block_table: torch.Tensor, row: int, seq_len: int) -> torch.Tensor:
    """Rows ``[0, seq_len)`` of one sequence from a paged cache ``[nb, bs, KH, D]``.

    Follows ``tests/test_paged_split_kv.py:34-36``: the physical pages are
    ``table[row, :ceil(L / bs)]`` and the flattened pages are truncated to L.
    """
    block_size = cache.shape[1]
    pages = block_table[row, : math.ceil(seq_len / block_size)].long()
    return cache[pages].reshape(-1, cache.shape[2], cache.shape[3])[:seq_len].float()


def paged_attention_reference(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    seqused_k: torch.Tensor,
    softmax_scale: float,
    out_dtype: torch.dtype | None = None,
    q_chunk: int | None = None,
) -> torch.Tensor:
    """Causal varlen paged attention in fp32 on the CPU.

    ``q`` is ``[T, H, D]``; ``k_cache``/``v_cache`` are ``[num_blocks, block_size,
    KH, D]`` views (the ``cache[:, 0]`` / ``cache[:, 1]`` of the reference test);
    ``cu_seqlens_q`` is ``[B + 1]`` and ``seqused_k`` ``[B]`` (total KV length
    including the new query tokens).  Returns ``[T, H, D]`` in ``out_dtype``
    (fp32 when ``None``).  ``q_chunk`` bounds host memory by processing query
    rows in chunks; the arithmetic per row is unchanged.
    """
    q = q.cpu()
    k_cache = k_cache.cpu()
    v_cache = v_cache.cpu()
    block_table = block_table.cpu()
    cu = [int(x) for x in cu_seqlens_q.cpu().tolist()]
    lens = [int(x) for x in seqused_k.cpu().tolist()]
    total, heads, dim = q.shape
    kv_heads = k_cache.shape[2]
    group = heads // kv_heads
    out = torch.zeros(total, heads, dim, dtype=torch.float32)
    for row, seq_len in enumerate(lens):
        q_begin, q_end = cu[row], cu[row + 1]
        q_len = q_end - q_begin
        if q_len <= 0 or seq_len <= 0:
            continue
        k = _gather_sequence_kv(k_cache, block_table, row, seq_len).repeat_interleave(group, dim=1)
        v = _gather_sequence_kv(v_cache, block_table, row, seq_len).repeat_interleave(group, dim=1)
        prefix = seq_len - q_len
        step = q_len if not q_chunk else q_chunk
        for c0 in range(0, q_len, step):
            c1 = min(q_len, c0 + step)
            qs = q[q_begin + c0 : q_begin + c1].float()
            logits = torch.einsum("qhd,khd->hqk", qs, k) * softmax_scale
            q_abs = prefix + torch.arange(c0, c1)
            causal = torch.arange(seq_len)[None, :] <= q_abs[:, None]
            logits.masked_fill_(~causal[None], float("-inf"))
            has_key = causal.any(dim=1)
            probs = torch.softmax(logits, dim=-1)
            probs = torch.where(has_key[None, :, None], probs, torch.zeros_like(probs))
            out[q_begin + c0 : q_begin + c1] = torch.einsum("hqk,khd->qhd", probs, v)
    if out_dtype is not None:
        return out.to(out_dtype)
    return out


def split_kv_partials_reference(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    seqused_k: torch.Tensor,
    softmax_scale: float,
    num_splits: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-split partial outputs ``(O_s, m_s, l_s)`` of ``_split_kv_forward``.

    Follows ``kernels/triton_split_kv_paged.py:69-79`` for the split ranges and
    query positions and ``:129-155`` for what is stored: ``O_s`` normalised by
    ``max(l_s, 1e-20)``, ``m_s`` the maximum scaled logit over the split's
    valid keys (``-inf`` if none), ``l_s = sum exp(logit - m_s)`` (0 if none).
    Shapes: ``O [S, T, H, D]`` fp32, ``m, l [S, T, H]`` fp32.
    """
    q = q.cpu()
    cu = [int(x) for x in cu_seqlens_q.cpu().tolist()]
    lens = [int(x) for x in seqused_k.cpu().tolist()]
    total, heads, dim = q.shape
    kv_heads = k_cache.shape[2]
    group = heads // kv_heads
    o_s = torch.zeros(num_splits, total, heads, dim)
    m_s = torch.full((num_splits, total, heads), float("-inf"))
    l_s = torch.zeros(num_splits, total, heads)
    for row, seq_len in enumerate(lens):
        q_begin, q_end = cu[row], cu[row + 1]
        q_len = q_end - q_begin
        if q_len <= 0 or seq_len <= 0:
            continue
        k = _gather_sequence_kv(k_cache.cpu(), block_table.cpu(), row, seq_len).repeat_interleave(group, dim=1)
        v = _gather_sequence_kv(v_cache.cpu(), block_table.cpu(), row, seq_len).repeat_interleave(group, dim=1)
        logits = torch.einsum("qhd,khd->hqk", q[q_begin:q_end].float(), k) * softmax_scale
        q_abs = seq_len - q_len + torch.arange(q_len)
        kv_pos = torch.arange(seq_len)
        split_size = (seq_len + num_splits - 1) // num_splits
        for s in range(num_splits):
            begin = s * split_size
            end = min(begin + split_size, seq_len)
            valid = (kv_pos[None, :] >= begin) & (kv_pos[None, :] < end) & (kv_pos[None, :] <= q_abs[:, None])
            masked = logits.masked_fill(~valid[None], float("-inf"))
            m = masked.max(dim=-1).values  # [H, q]
            has = valid.any(dim=1)[None, :].expand_as(m)
            safe = torch.where(has, m, torch.zeros_like(m))
            p = torch.exp(masked - safe[..., None])
            l = p.sum(dim=-1)
            o = torch.einsum("hqk,khd->qhd", p, v) / torch.clamp(l, min=1e-20).transpose(0, 1)[..., None]
            o_s[s, q_begin:q_end] = o
            m_s[s, q_begin:q_end] = torch.where(has, m, torch.full_like(m, float("-inf"))).transpose(0, 1)
            l_s[s, q_begin:q_end] = l.transpose(0, 1)
    return o_s, m_s, l_s


def split_kv_reduce_reference(o_splits: torch.Tensor, m_splits: torch.Tensor, l_splits: torch.Tensor) -> torch.Tensor:
    """Cross-split combine of ``_split_kv_reduce`` (``kernels/triton_split_kv_paged.py:197-228``).

    ``o_splits [S, T, H, D]`` (any float dtype, read as fp32), ``m_splits`` and
    ``l_splits [S, T, H]`` fp32.  Returns ``[T, H, D]`` fp32.
    """
    o = o_splits.float().cpu()
    m = m_splits.float().cpu()
    l = l_splits.float().cpu()
    m_global = m.max(dim=0).values
    active = l > 0
    safe_global = torch.where(torch.isfinite(m_global), m_global, torch.zeros_like(m_global))
    weight = torch.where(active, torch.exp(m - safe_global[None]) * l, torch.zeros_like(l))
    o = torch.where(active[..., None], o, torch.zeros_like(o))
    acc = (weight[..., None] * o).sum(dim=0)
    denom = weight.sum(dim=0)
    return acc / torch.clamp(denom, min=1e-20)[..., None]
