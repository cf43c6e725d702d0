"""Seeded synthetic batches for the paged attention and RoPE/KV-write paths.

Every tensor is drawn on the CPU from ``torch.Generator`` streams so that the
GPU kernels and the CPU checker see identical bytes.  Values are drawn in
fp32 and rounded to the storage dtype once; the checker reads the rounded
values.

The batch layout follows the reference's own builders
(``tests/test_paged_split_kv.py:59-82`` and ``tests/attention_harness.py:73-115``):
a paged cache ``[num_blocks, 2, block_size, KV_heads, D]`` (K at ``[:, 0]``,
V at ``[:, 1]``), a block table whose rows list each sequence's physical pages
(a seeded random permutation of the pool, so kernels that assume consecutive
pages fail), ``cu_seqlens_q [B + 1]`` and ``seqused_k [B]`` in int32.

Per-sequence content (query rows and that sequence's logical pages) comes from
a generator keyed on ``(seed, sequence index)``, so a shard of sequences can be
built on its own (one process per GPU) and still holds the same values as the
same sequences in the full batch.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import torch

DEFAULT_SEED = 20260928  # the seed of tests/test_paged_split_kv.py:110 in the reference

NUM_Q_HEADS = 16
NUM_KV_HEADS = 2
HEAD_DIM = 128
BLOCK_SIZE = 16


def _gen(*keys: int) -> torch.Generator:
    """A CPU generator keyed on a tuple of integers."""
    h = 0x9E3779B97F4A7C15
    for k in keys:
        h = (h ^ (int(k) & 0xFFFFFFFFFFFFFFFF)) * 0xBF58476D1CE4E5B9 & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 31
    return torch.Generator().manual_seed(h & 0x7FFFFFFFFFFFFFFF)


@dataclass
class AttentionBatch:
    q: torch.Tensor  # [T, H, D]
    kv_cache: torch.Tensor  # [num_blocks, 2, block_size, KH, D]
    block_table: torch.Tensor  # [B, max_pages] int32
    cu_seqlens_q: torch.Tensor  # [B + 1] int32
    seqused_k: torch.Tensor  # [B] int32
    query_lens: list[int]
    kv_lens: list[int]
    softmax_scale: float
    seq_ids: list[int]

    @property
    def k_cache(self) -> torch.Tensor:
        return self.kv_cache[:, 0]

    @property
    def v_cache(self) -> torch.Tensor:
        return self.kv_cache[:, 1]

    @property
    def max_seqlen_q(self) -> int:
        return max(self.query_lens) if self.query_lens else 0

    @property
    def max_seqlen_k(self) -> int:
        return max(self.kv_lens) if self.kv_lens else 0

    @property
    def total_q(self) -> int:
        return int(self.q.shape[0])

    def to(self, device) -> "AttentionBatch":
        return AttentionBatch(
            q=self.q.to(device),
            kv_cache=self.kv_cache.to(device),
            block_table=self.block_table.to(device),
            cu_seqlens_q=self.cu_seqlens_q.to(device),
            seqused_k=self.seqused_k.to(device),
            query_lens=list(self.query_lens),
            kv_lens=list(self.kv_lens),
            softmax_scale=self.softmax_scale,
            seq_ids=list(self.seq_ids),
        )


def build_attention_batch(
    query_lens: Sequence[int],
    kv_lens: Sequence[int],
    *,
    seed: int = DEFAULT_SEED,
    num_q_heads: int = NUM_Q_HEADS,
    num_kv_heads: int = NUM_KV_HEADS,
    head_dim: int = HEAD_DIM,
    block_size: int = BLOCK_SIZE,
    pool_pages: int | None = None,
    dtype: torch.dtype = torch.bfloat16,
    seq_ids: Sequence[int] | None = None,
    permute: bool = True,
    extra_table_cols: int = 0,
) -> AttentionBatch:
    """Build one paged batch.

    ``kv_lens`` are total KV lengths (prior context + the query chunk), the
    ``seqused_k`` of the ABI.  ``seq_ids`` name the sequences' positions in a
    larger batch (default ``0..B-1``); content is keyed on them.
    """
    assert len(query_lens) == len(kv_lens)
    seq_ids = list(range(len(query_lens))) if seq_ids is None else list(seq_ids)
    pages = [math.ceil(L / block_size) for L in kv_lens]
    needed = sum(pages)
    pool = max(needed, pool_pages or 0, 1)
    layout_gen = _gen(seed, 7, *seq_ids[:4], len(seq_ids), pool)
    perm = torch.randperm(pool, generator=layout_gen) if permute else torch.arange(pool)
    cache = torch.empty(pool, 2, block_size, num_kv_heads, head_dim, dtype=dtype)
    if pool > needed:
        # Unused pool pages hold noise too: a kernel that reads a wrong page sees wrong values.
        cache[perm[needed:]] = torch.randn(pool - needed, 2, block_size, num_kv_heads, head_dim, generator=layout_gen).to(dtype)
    width = max(max(pages) if pages else 1, 1) + extra_table_cols
    table = torch.zeros(len(query_lens), width, dtype=torch.int32)
    qs = []
    nxt = 0
    for row, (sid, q_len, n) in enumerate(zip(seq_ids, query_lens, pages)):
        phys = perm[nxt : nxt + n]
        nxt += n
        table[row, :n] = phys.to(torch.int32)
        if n:
            cache[phys.long()] = torch.randn(n, 2, block_size, num_kv_heads, head_dim, generator=_gen(seed, 1, sid)).to(dtype)
        qs.append(torch.randn(q_len, num_q_heads, head_dim, generator=_gen(seed, 0, sid)).to(dtype))
    q = torch.cat(qs) if qs else torch.empty(0, num_q_heads, head_dim, dtype=dtype)
    cu = torch.tensor([0, *torch.tensor(list(query_lens), dtype=torch.int64).cumsum(0).tolist()], dtype=torch.int32)
    return AttentionBatch(
        q=q,
        kv_cache=cache,
        block_table=table,
        cu_seqlens_q=cu,
        seqused_k=torch.tensor(list(kv_lens), dtype=torch.int32),
        query_lens=list(query_lens),
        kv_lens=list(kv_lens),
        softmax_scale=1.0 / math.sqrt(head_dim),
        seq_ids=seq_ids,
    )


# ---------------------------------------------------------------------------
# The five workload shapes of the attention and RoPE paths.
# ---------------------------------------------------------------------------

def lengths_correctness() -> tuple[list[int], list[int]]:
    """4 sequences, query lengths [37, 128, 255, 64] over prior context [0, 300, 1000, 2047]."""
    q = [37, 128, 255, 64]
    prior = [0, 300, 1000, 2047]
    return q, [p + x for p, x in zip(prior, q)]


def lengths_chunked_4k(seed: int = DEFAULT_SEED, num_seqs: int = 64) -> tuple[list[int], list[int]]:
    """64 sequences, 512-token query chunks, total KV length uniform in [1024, 4096]."""
    g = _gen(seed, 4096)
    kv = torch.randint(1024, 4096 + 1, (num_seqs,), generator=g).tolist()
    return [512] * num_seqs, kv


def lengths_chunked_16k(seed: int = DEFAULT_SEED, num_seqs: int = 64) -> tuple[list[int], list[int]]:
    """64 sequences, 2048-token query chunks, total KV length uniform in [8192, 16384]."""
    g = _gen(seed, 16384)
    kv = torch.randint(8192, 16384 + 1, (num_seqs,), generator=g).tolist()
    return [2048] * num_seqs, kv


def lengths_mixed(seed: int = DEFAULT_SEED, num_seqs: int = 256) -> tuple[list[int], list[int]]:
    """256 sequences: half decode rows (q = 1), half q uniform in [16, 1024]; KV uniform in [512, 16384]."""
    g = _gen(seed, 256)
    decode = torch.rand(num_seqs, generator=g) < 0.5
    qlen = torch.randint(16, 1024 + 1, (num_seqs,), generator=g)
    qlen = torch.where(decode, torch.ones_like(qlen), qlen)
    kv = torch.randint(512, 16384 + 1, (num_seqs,), generator=g)
    kv = torch.maximum(kv, qlen)
    return qlen.tolist(), kv.tolist()


def lengths_decode_16k(seed: int = DEFAULT_SEED, num_seqs: int = 64) -> tuple[list[int], list[int]]:
    """64 decode rows (one new token each), total KV length uniform in [8192, 16384]."""
    g = _gen(seed, 16384, 1)
    kv = torch.randint(8192, 16384 + 1, (num_seqs,), generator=g).tolist()
    return [1] * num_seqs, kv


def lengths_decode_4k(seed: int = DEFAULT_SEED, num_seqs: int = 256) -> tuple[list[int], list[int]]:
    """256 decode rows, total KV length uniform in [1024, 4096]."""
    g = _gen(seed, 4096, 1)
    kv = torch.randint(1024, 4096 + 1, (num_seqs,), generator=g).tolist()
    return [1] * num_seqs, kv


WORKLOADS = {
    "correctness": lengths_correctness,
    "chunked_prefill_4k": lengths_chunked_4k,
    "chunked_prefill_16k": lengths_chunked_16k,
    "mixed_256": lengths_mixed,
    "decode_16k": lengths_decode_16k,
    "decode_4k": lengths_decode_4k,
}


def attention_kv_bytes(query_lens: Sequence[int], kv_lens: Sequence[int], num_kv_heads: int = 2,
                       head_dim: int = 128, elem: int = 2, num_q_heads: int = 16) -> int:
    """Bytes one pass must move at minimum: every K and V row of every sequence once, Q read, O written."""
    kv = 2 * sum(kv_lens) * num_kv_heads * head_dim * elem
    qo = 2 * sum(query_lens) * num_q_heads * head_dim * elem
    return kv + qo


def correctness_batch(seed: int = DEFAULT_SEED, dtype: torch.dtype = torch.bfloat16) -> AttentionBatch:
    """The CPU-checkable case: 4 sequences in a pool of 512 pages (241 used)."""
    q, kv = lengths_correctness()
    return build_attention_batch(q, kv, seed=seed, pool_pages=512, dtype=dtype)


# ---------------------------------------------------------------------------
# RoPE + KV-cache write inputs.
# ---------------------------------------------------------------------------

@dataclass
class RopeBatch:
    query: torch.Tensor  # [T, Hq, D]
    key: torch.Tensor  # [T, Hkv, D]
    value: torch.Tensor  # [T, Hkv, D]
    positions: torch.Tensor  # [T]
    cos_sin_cache: torch.Tensor  # [max_pos, rotary_dim]
    key_cache: torch.Tensor  # [num_blocks, block_size, Hkv, D]
    value_cache: torch.Tensor
    slot_mapping: torch.Tensor  # [T]
    is_neox: bool
    rotary_dim: int

    def to(self, device) -> "RopeBatch":
        return RopeBatch(**{k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()})

    def clone(self) -> "RopeBatch":
        return RopeBatch(**{k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()})


def rope_cos_sin(max_position: int, rotary_dim: int, base: float = 10000.0, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``[max_position, rotary_dim]`` table ``[cos | sin]`` with ``inv_freq = base^(-2i / rd)``."""
    inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim))
    t = torch.arange(max_position, dtype=torch.float64)
    freqs = torch.outer(t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(dtype)


def build_rope_batch(
    tokens: int = 16384,
    *,
    rotary_dim: int = 128,
    is_neox: bool = True,
    num_q_heads: int = NUM_Q_HEADS,
    num_kv_heads: int = NUM_KV_HEADS,
    head_dim: int = HEAD_DIM,
    block_size: int = BLOCK_SIZE,
    num_blocks: int = 4096,
    max_position: int = 16384,
    seed: int = DEFAULT_SEED,
    dtype: torch.dtype = torch.bfloat16,
    pos_dtype: torch.dtype = torch.int64,
    slot_dtype: torch.dtype = torch.int64,
    sentinel: float = 7.0,
) -> RopeBatch:
    """16384 new tokens at random positions, scattered by a seeded injection into the cache."""
    g = _gen(seed, 31, tokens, rotary_dim, int(is_neox))
    query = torch.randn(tokens, num_q_heads, head_dim, generator=g).to(dtype)
    key = torch.randn(tokens, num_kv_heads, head_dim, generator=g).to(dtype)
    value = torch.randn(tokens, num_kv_heads, head_dim, generator=g).to(dtype)
    positions = torch.randint(0, max_position, (tokens,), generator=g).to(pos_dtype)
    slots = torch.randperm(num_blocks * block_size, generator=g)[:tokens].to(slot_dtype)
    key_cache = torch.full((num_blocks, block_size, num_kv_heads, head_dim), sentinel, dtype=dtype)
    value_cache = torch.full_like(key_cache, -sentinel)
    return RopeBatch(
        query=query,
        key=key,
        value=value,
        positions=positions,
        cos_sin_cache=rope_cos_sin(max_position, rotary_dim, dtype=dtype),
        key_cache=key_cache,
        value_cache=value_cache,
        slot_mapping=slots,
        is_neox=is_neox,
        rotary_dim=rotary_dim,
    )


def rope_algorithmic_bytes(b: RopeBatch) -> int:
    """Bytes the RoPE + cache write must move at minimum.

    The rotated part of Q read + written (Q's dims past ``rotary_dim`` are
    left in place and need not move), K and V read, K and V cache rows written,
    one cos/sin row read per token, positions and slots read.  Tokens with
    ``slot < 0`` move no cache bytes.
    """
    t, hq, d = b.query.shape
    hkv = b.key.shape[1]
    e = b.query.element_size()
    written = int((b.slot_mapping >= 0).sum())
    q_bytes = 2 * t * hq * b.rotary_dim * e
    kv_read = 2 * t * hkv * d * e
    kv_write = 2 * written * hkv * d * e
    cs = t * b.rotary_dim * b.cos_sin_cache.element_size()
    idx = t * (b.positions.element_size() + b.slot_mapping.element_size())
    return q_bytes + kv_read + kv_write + cs + idx


# ---------------------------------------------------------------------------
# Paged KV-cache write (the service's cache update).
# ---------------------------------------------------------------------------

# kv_cache_dtype string -> (cache torch dtype, inline scale padding in elements)
KV_CACHE_KINDS = {
    "auto": (None, 0),
    "fp8": (torch.float8_e4m3fn, 0),
    "int8_per_token_head": (torch.int8, 4),
    "fp8_per_token_head": (torch.float8_e4m3fn, 4),
}


@dataclass
class KvWriteBatch:
    key: torch.Tensor  # [T, KH, D]
    value: torch.Tensor  # [T, KH, D]
    slot_mapping: torch.Tensor  # [T]; negative = padding token
    kv_cache: torch.Tensor  # [num_blocks, 2, block_size, KH, D + pad], sentinel-filled
    kv_cache_dtype: str
    k_scale: torch.Tensor  # [1] float32 (fp8 per-tensor)
    v_scale: torch.Tensor

    def to(self, device) -> "KvWriteBatch":
        return KvWriteBatch(**{k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()})

    def clone(self) -> "KvWriteBatch":
        return KvWriteBatch(**{k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in self.__dict__.items()})

    @property
    def head_dim(self) -> int:
        return self.key.shape[2]

    def caches(self) -> tuple[torch.Tensor, torch.Tensor]:
        """``kv_cache.unbind(1)`` trimmed to head_dim: the data part of each cache row."""
        k, v = self.kv_cache.unbind(1)
        d = self.head_dim
        return k[..., :d], v[..., :d]

    def scale_cache_views(self) -> tuple[torch.Tensor, torch.Tensor]:
        """float32 views ``[num_blocks, block_size, KH]`` of the inline per-token-head scales.

        The scale of (block, slot, head) is the float32 in the 4 bytes after
        head_dim of that cache row, as the service's ``_ensure_scale_caches``
        lays it out (integration/vllm-plugin-FL-split-kv.patch:473-523).
        """
        nb, _, bs, kh, padded = self.kv_cache.shape
        e = self.kv_cache.element_size()
        row = padded * e
        assert row % 4 == 0 and (self.kv_cache.storage_offset() * e) % 4 == 0
        base = torch.empty(0, dtype=torch.float32, device=self.kv_cache.device).set_(self.kv_cache.untyped_storage())
        half = bs * kh * row
        start = self.kv_cache.storage_offset() * e // 4 + self.head_dim * e // 4
        stride = (2 * half // 4, kh * row // 4, row // 4)
        ks = torch.as_strided(base, (nb, bs, kh), stride, start)
        vs = torch.as_strided(base, (nb, bs, kh), stride, start + half // 4)
        return ks, vs


def build_kv_write_batch(
    tokens: int = 16384,
    *,
    kv_cache_dtype: str = "auto",
    num_kv_heads: int = NUM_KV_HEADS,
    head_dim: int = HEAD_DIM,
    block_size: int = BLOCK_SIZE,
    num_blocks: int = 4096,
    padding_tokens: int = 0,
    seed: int = DEFAULT_SEED,
    dtype: torch.dtype = torch.bfloat16,
    slot_dtype: torch.dtype = torch.int64,
    k_scale: float = 0.0125,
    v_scale: float = 0.0089,
) -> KvWriteBatch:
    """New K/V rows scattered by a seeded injection into a sentinel-filled 5-D cache.

    Values are N(0, 1) with every 16th (token, head) row scaled by 20 so the
    per-token-head scales vary and the per-tensor fp8 path meets saturation.
    The last ``padding_tokens`` tokens get slot -1.
    """
    g = _gen(seed, 47, tokens, num_kv_heads, head_dim, len(kv_cache_dtype))
    boost = torch.ones(tokens, num_kv_heads, 1)
    boost.view(-1)[::16] = 20.0
    key = (torch.randn(tokens, num_kv_heads, head_dim, generator=g) * boost).to(dtype)
    value = (torch.randn(tokens, num_kv_heads, head_dim, generator=g) * boost.flip(0)).to(dtype)
    slots = torch.randperm(num_blocks * block_size, generator=g)[:tokens]
    if padding_tokens:
        slots[tokens - padding_tokens :] = -1
    cache_dtype, pad = KV_CACHE_KINDS[kv_cache_dtype]
    cache_dtype = cache_dtype or dtype
    shape = (num_blocks, 2, block_size, num_kv_heads, head_dim + pad)
    if cache_dtype in (torch.int8, torch.float8_e4m3fn):
        kv_cache = torch.full(shape, 0x5A, dtype=torch.uint8).view(cache_dtype)
    else:
        kv_cache = torch.full(shape, 7.0, dtype=cache_dtype)
    return KvWriteBatch(
        key=key,
        value=value,
        slot_mapping=slots.to(slot_dtype),
        kv_cache=kv_cache,
        kv_cache_dtype=kv_cache_dtype,
        k_scale=torch.tensor([k_scale], dtype=torch.float32),
        v_scale=torch.tensor([v_scale], dtype=torch.float32),
    )


def kv_write_algorithmic_bytes(b: KvWriteBatch) -> int:
    """K and V read, K and V cache rows (plus per-token-head scales) written, slots read."""
    t, kh, d = b.key.shape
    written = int((b.slot_mapping >= 0).sum())
    read = 2 * t * kh * d * b.key.element_size()
    write = 2 * written * kh * d * b.kv_cache.element_size()
    if b.kv_cache_dtype.endswith("per_token_head"):
        write += 2 * written * kh * 4
    return read + write + t * b.slot_mapping.element_size()
