"""Golden vectors for the paged KV-cache write, from vLLM's own Triton kernels.

The service's cache update (``IluvatarAttentionImpl.do_kv_cache_update`` in
``integration/vllm-plugin-FL-split-kv.patch:815-858`` of the reference
project) calls vLLM's ``triton_reshape_and_cache_flash`` and
``triton_reshape_and_cache_flash_per_token_head_quant``.  This script runs
those kernels on the CPU under ``TRITON_INTERPRET=1`` on small seeded batches
and stores what they wrote.

Cases: "auto" caches in bf16, fp16 and fp32, and the int8 per-token-head
cache.  fp8 caches are not generated: the interpreter's float -> fp8
conversion does not round to nearest (e.g. 126.2 -> 64), so its fp8 output
is not the GPU kernel's; the fp8 encoder of the oracle is pinned instead
against torch's conversion over every bf16 value, and the GPU tests compare
the fp8 caches with vLLM's kernel running on the GPU.

The wrapper of vLLM 0.22 asks torch for the device's compute capability; with
no GPU here it is answered as 10.0 (sm_100), which selects the CUDA launch
parameters.  The per-token-head scales go to separate (unaliased) tensors:
the interpreter copies each argument, so aliasing views would not be written
back reliably.

Inputs are rebuilt by ``minicpm_b200.workloads.build_kv_write_batch`` and
checked by sha256.

Usage (needs vLLM importable; no GPU)::

    python tests/golden/make_kv_golden.py
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "minicpm-attention-optimization-iluvatar_b200"))

from minicpm_b200 import workloads  # noqa: E402

# name, kv_cache_dtype, model dtype, tokens, kv_heads, head_dim, blocks, padding tokens
KV_CASES = [
    ("auto_bf16", "auto", torch.bfloat16, 96, 2, 128, 16, 5),
    ("auto_fp16", "auto", torch.float16, 40, 4, 64, 8, 3),
    ("auto_fp32", "auto", torch.float32, 33, 1, 256, 4, 0),
    ("int8_pth_bf16", "int8_per_token_head", torch.bfloat16, 96, 2, 128, 16, 5),
    ("int8_pth_fp16", "int8_per_token_head", torch.float16, 40, 4, 64, 8, 3),
]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def batch_for(case) -> workloads.KvWriteBatch:
    _, kind, dtype, tokens, kh, d, blocks, pad = case
    return workloads.build_kv_write_batch(
        tokens, kv_cache_dtype=kind, num_kv_heads=kh, head_dim=d, num_blocks=blocks, padding_tokens=pad, dtype=dtype
    )


def run_case(case) -> dict:
    torch.cuda.get_device_capability = lambda *a, **k: (10, 0)
    from vllm.v1.attention.ops import triton_reshape_and_cache_flash as vk

    b = batch_for(case)
    _, kind, dtype, tokens, kh, d, blocks, pad = case
    rec = {"kind": np.array(kind), "dtype": np.array(str(dtype).replace("torch.", "")),
           "dims": np.array([tokens, kh, d, blocks, pad], np.int64)}
    rec |= {"sha_key": np.array(sha(b.key)), "sha_value": np.array(sha(b.value)), "sha_slots": np.array(sha(b.slot_mapping))}
    kc, vc = b.caches()
    slots = b.slot_mapping.long()
    idx = torch.nonzero(slots >= 0).flatten()
    blk, off = slots[idx] // kc.shape[1], slots[idx] % kc.shape[1]
    if b.kv_cache_dtype == "auto":
        vk.triton_reshape_and_cache_flash(b.key, b.value, kc, vc, b.slot_mapping, "auto", b.k_scale, b.v_scale)
    else:
        nb, bs, kh, _ = kc.shape
        ksc = torch.zeros(nb, bs, kh)
        vsc = torch.zeros(nb, bs, kh)
        vk.triton_reshape_and_cache_flash_per_token_head_quant(b.key, b.value, kc, vc, ksc, vsc, b.slot_mapping)
        rec["k_scale_rows"] = ksc[blk, off].numpy()
        rec["v_scale_rows"] = vsc[blk, off].numpy()
    rec["k_rows"] = kc[blk, off].contiguous().view(torch.uint8).numpy()
    rec["v_rows"] = vc[blk, off].contiguous().view(torch.uint8).numpy()
    return rec


def main() -> None:
    out = {}
    for case in KV_CASES:
        for k, v in run_case(case).items():
            out[f"{case[0]}__{k}"] = v
        print("ran", case[0], flush=True)
    np.savez_compressed(HERE / "kv_write_vllm_cases.npz", **out)
    print("wrote kv_write_vllm_cases.npz")


if __name__ == "__main__":
    main()
