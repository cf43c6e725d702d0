"""fp32 CPU restatement of the reference's fused RoPE + paged KV-cache write.

TEST INFRASTRUCTURE ONLY (the checker and the CPU baseline; never shipped).

Reference files followed (paths inside the reference project):

* ``tests/test_rope_kv_cache.py:17-32`` -- ``reference_rope``: the rotation in
  fp32 from ``cos_sin_cache[pos] = [cos(0..half) | sin(0..half)]``; NeoX pairs
  ``(d, d + half)``, interleaved pairs ``(2i, 2i + 1)``; dims at or beyond
  ``rotary_dim`` pass through; result cast back to the input dtype.
* ``kernels/triton_rope_kv_cache.py:53-55,114-115,181-202`` -- what is written
  where: Q is rotated in place for every token (also when ``slot < 0``); the
  rotated K goes to ``key_cache[slot // bs, slot % bs, h, :]`` and V is copied
  unchanged to ``value_cache[...]``; both writes are skipped when ``slot < 0``;
  the input ``key``/``value`` tensors are not modified.

The products ``x * cos`` and ``partner * sin`` are rounded separately and then
added (no fused multiply-add), which is what the torch expression in
``tests/test_rope_kv_cache.py:24-29`` computes.
"""

from __future__ import annotations

import torch


def rotate_fp32(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor, is_neox: bool, rotary_dim: int) -> torch.Tensor:
    """The fp32 rotation of ``x [T, heads, D]`` before the cast back to storage dtype.

    Restates ``tests/test_rope_kv_cache.py:18-31``.
    """
    out = x.detach().cpu().clone().float()
    half = rotary_dim // 2
    cos, sin = cos_sin.cpu()[positions.cpu().long()].float().split(half, dim=-1)
    cos = cos[:, None, :]
    sin = sin[:, None, :]
    rot = out[..., :rotary_dim]
    if is_neox:
        first, second = rot[..., :half], rot[..., half:rotary_dim]
        rotated = torch.cat((first * cos - second * sin, first * sin + second * cos), dim=-1)
    else:
        even, odd = rot[..., 0::2], rot[..., 1::2]
        rotated = torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1).flatten(-2)
    out[..., :rotary_dim] = rotated
    return out


def reference_rope(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor, is_neox: bool, rotary_dim: int) -> torch.Tensor:
    """Rotate ``x [T, heads, D]`` by the rows ``cos_sin[positions]``; same dtype out.

    Restates ``tests/test_rope_kv_cache.py:17-32``; the cast rounds to nearest
    even, as the GPU store of the reference kernel does.
    """
    return rotate_fp32(x, cos_sin, positions, is_neox, rotary_dim).to(x.dtype)


def rope_and_cache_reference(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    is_neox: bool,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    rotary_dim: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Expected ``(query, key_cache, value_cache)`` after ``fused_rope_and_cache``.

    Works on CPU copies and returns new tensors; the inputs are not modified.
    ``key_cache``/``value_cache`` are ``[num_blocks, block_size, KH, D]``.
    """
    rotary_dim = rotary_dim or int(cos_sin_cache.shape[1])
    q_out = reference_rope(query, cos_sin_cache, positions, is_neox, rotary_dim)
    k_rot = reference_rope(key, cos_sin_cache, positions, is_neox, rotary_dim)
    kc = key_cache.detach().cpu().clone()
    vc = value_cache.detach().cpu().clone()
    block_size = kc.shape[1]
    slots = slot_mapping.cpu().long()
    keep = slots >= 0
    idx = torch.nonzero(keep).flatten()
    blocks = torch.div(slots[idx], block_size, rounding_mode="floor")
    offsets = slots[idx] - blocks * block_size
    kc[blocks, offsets] = k_rot[idx].to(kc.dtype)
    vc[blocks, offsets] = value.detach().cpu()[idx].to(vc.dtype)
    return q_out, kc, vc
