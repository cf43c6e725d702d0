"""sm_100a (B200) paged prefill attention and fused RoPE + KV-cache write.

The operator API of the reference's ``kernels`` package, backed by
hand-written CUDA in ``libminicpm_b200.so``:

* :func:`iluvatar_attention` -- the vLLM-ABI dispatcher (``kernels/attention.py``)
* :func:`unified_attention_optimized` -- the launch-policy shim
  (``kernels/triton_unified_attention_optimized.py``)
* :func:`paged_split_kv_attention` -- paged Split-KV causal attention
  (``kernels/triton_split_kv_paged.py``)
* :func:`fused_rope_and_cache` -- fused RoPE + paged KV-cache write
  (``kernels/triton_rope_kv_cache.py``)
"""

from .attention import iluvatar_attention
from .rope_kv_cache import fused_rope_and_cache
from .split_kv_paged import choose_num_splits, paged_split_kv_attention, split_kv_combine
from .unified_attention_optimized import unified_attention_optimized

__all__ = [
    "iluvatar_attention",
    "unified_attention_optimized",
    "paged_split_kv_attention",
    "split_kv_combine",
    "choose_num_splits",
    "fused_rope_and_cache",
]
