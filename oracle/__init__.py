"""CPU oracle for the paged prefill attention and RoPE + KV-cache write path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory.  It is used by ``tests/``, by ``__graft_entry__.smoke()`` as the
checker, and by ``bench.py`` for the timed CPU baseline leg only.

Every function restates the algorithm of the reference implementation in
plain fp32 torch/numpy on the CPU and cites the reference file and lines it
follows.  The restatement is pinned against golden vectors produced by the
reference's own Triton kernels run under ``TRITON_INTERPRET=1`` on the CPU
(``tests/golden/make_golden.py``; fixtures in ``tests/golden/*.npz``), and,
for the service's KV-cache writes, by vLLM's Triton kernels run the same way
(``tests/golden/make_kv_golden.py``).
"""

from .paged_sdpa import (
    causal_flops,
    paged_attention_reference,
    split_kv_partials_reference,
    split_kv_reduce_reference,
)
from .kv_cache import (
    dequantize_cache_reference,
    fp8_decode,
    fp8_encode,
    kv_write_reference,
    quantize_per_tensor,
    quantize_per_token_head,
    rope_and_cache_service_reference,
)
from .rope import reference_rope, rope_and_cache_reference, rotate_fp32

__all__ = [
    "causal_flops",
    "paged_attention_reference",
    "split_kv_partials_reference",
    "split_kv_reduce_reference",
    "reference_rope",
    "rope_and_cache_reference",
    "rotate_fp32",
    "fp8_encode",
    "dequantize_cache_reference",
    "fp8_decode",
    "quantize_per_tensor",
    "quantize_per_token_head",
    "kv_write_reference",
    "rope_and_cache_service_reference",
]
