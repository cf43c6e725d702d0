"""The serving backend of the reference (its vLLM plugin shim) on the sm_100a operators.

Mirrors ``vllm_fl/dispatch/backends/vendor/iluvatar/impl/attention.py`` as the
reference's integration patch adds it (``integration/vllm-plugin-FL-split-kv.patch``):

* :func:`_run_unified_attention` (patch :88-141) -- the per-call route: the
  sm_100a Split-KV path when ``ILUVATAR_USE_OPTIMIZED`` and
  ``ILUVATAR_SPLIT_KV`` are both set ("1", "true" or "yes") and the call uses
  no unsupported feature (ALiBi, sinks, softcap, a sliding window, a query
  descale or a descale without an fp8 per-tensor cache, nvfp4, tensor
  descriptors, non-causal), else vLLM's
  ``unified_attention``.  A head shape or dtype the sm_100a kernel does not
  run (``kernel_supports``: fp32, head_dim other than 64 / 128 / 256, more than
  128 query heads per KV head) takes the vLLM route too.  Pure decode (``max_seqlen_q <= 1``) stays on vLLM
  unless ``ILUVATAR_SPLIT_KV_DECODE`` is also set, which selects the sm_100a
  decode kernel (the reference kept decode on vLLM).  Failures of the sm_100a
  path propagate; there is no silent fallback.
* :class:`IluvatarAttentionImpl` (patch :468-899) -- ``forward`` (profiling run,
  encoder attention, per-token-head and fp8 caches, the call above),
  ``do_kv_cache_update`` (the sm_100a cache writers of :mod:`.kv_cache`) and
  ``do_rope_and_kv_cache_update`` (the fused RoPE + cache write).
* :class:`IluvatarAttentionMetadata`, :class:`IluvatarAttentionMetadataBuilder`
  and :class:`IluvatarAttentionBackend` (patch :150-466) -- the metadata, its
  builder and the backend's static contract (cache shape and stride order,
  supported dtypes and block sizes).

Differences from the reference, on purpose:

* Quantised caches (fp8 per-tensor, int8 / fp8 per-token-head) take the
  sm_100a path: the pages a call references are dequantised into a dense cache
  in the query dtype (``b200_kv_dequant_pages``), then the same attention
  kernel runs.  The reference sends every quantised cache to vLLM.

* The k/v-descale guard.  For unquantised (auto / bf16 / fp16) caches the
  reference's ``forward`` passes ``layer._k_scale.expand(...)`` and
  ``layer._v_scale.expand(...)`` as ``k_descale`` / ``v_descale``, and the
  route treats any descale as unsupported, so the optimized path was never
  taken in the service (``docs/stage-summary-2026-10-09.md``, section 6).  Here
  the descales are passed only when the cache is quantised.
* ``ILUVATAR_NUM_SPLITS`` unset means an automatically chosen split count
  (the reference used 4).
* ``fused_rope_kvcache_supported`` is true for every cache except the
  per-token-head ones: the fused RoPE + cache write exists here (the
  reference's depended on ROCm's aiter and was off on other platforms).
* The builder and backend are plain classes with the same fields and
  methods; they take the model sizes directly instead of a vLLM config.

vLLM is imported only for the routes that stay on vLLM (its
``unified_attention`` and ``context_attention_fwd``); ``RuntimeError`` is raised
there when it is not installed.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from enum import IntEnum
from typing import Any, ClassVar

import torch

from .kv_cache import (
    is_quantized_kv_cache,
    reshape_and_cache_flash,
    reshape_and_cache_flash_per_token_head_quant,
    rope_and_cache,
)
from .split_kv_paged import kernel_supports
from .unified_attention_optimized import unified_attention_optimized


class KVQuantMode(IntEnum):
    """vLLM's KV-cache quantisation modes (``vllm/v1/kv_cache_interface.py``)."""

    NONE = 0
    FP8_PER_TENSOR = 1
    INT8_PER_TOKEN_HEAD = 2
    FP8_PER_TOKEN_HEAD = 3
    NVFP4 = 4

    @property
    def is_per_token_head(self) -> bool:
        return self in (KVQuantMode.INT8_PER_TOKEN_HEAD, KVQuantMode.FP8_PER_TOKEN_HEAD)


def get_kv_quant_mode(kv_cache_dtype: str) -> KVQuantMode:
    if kv_cache_dtype == "int8_per_token_head":
        return KVQuantMode.INT8_PER_TOKEN_HEAD
    if kv_cache_dtype == "fp8_per_token_head":
        return KVQuantMode.FP8_PER_TOKEN_HEAD
    if kv_cache_dtype == "nvfp4":
        return KVQuantMode.NVFP4
    if kv_cache_dtype.startswith("fp8"):
        return KVQuantMode.FP8_PER_TENSOR
    return KVQuantMode.NONE


class AttentionType:
    DECODER = "decoder"
    ENCODER = "encoder"
    ENCODER_ONLY = "encoder_only"
    ENCODER_DECODER = "encoder_decoder"


FP8_DTYPE = torch.float8_e4m3fn
MIN_LAUNCH_GRID_SIZE_2D = 128  # vLLM's 2D/3D kernel threshold (only its baseline uses it)
NUM_PAR_SOFTMAX_SEGMENTS = 16


def _flag(name: str) -> bool:
    return os.environ.get(name, "0").lower() in ("1", "true", "yes")


def _vllm_unified_attention():
    try:
        from vllm.v1.attention.ops.triton_unified_attention import unified_attention
    except Exception as exc:  # vLLM missing or broken
        raise RuntimeError(f"this call stays on vLLM's unified_attention, which is unavailable: {exc}") from exc
    return unified_attention


def _run_unified_attention(**kwargs: Any) -> torch.Tensor:
    """Use the sm_100a path for supported prefill / mixed (and, if enabled, decode) calls."""
    enabled = _flag("ILUVATAR_USE_OPTIMIZED") and _flag("ILUVATAR_SPLIT_KV")
    max_query_len = kwargs["max_seqlen_q"]
    mode = KVQuantMode(int(kwargs.get("kv_quant_mode", KVQuantMode.NONE)))
    # Descales belong to the fp8 per-tensor cache (its dequantisation scales);
    # with any other cache they are a feature the sm_100a path does not have.
    descaled = kwargs.get("k_descale") is not None or kwargs.get("v_descale") is not None
    unsupported = (
        mode == KVQuantMode.NVFP4
        or (mode == KVQuantMode.FP8_PER_TENSOR and not (kwargs.get("k_descale") is not None
                                                       and kwargs.get("v_descale") is not None))
        or (mode.is_per_token_head and (kwargs.get("k_scale_cache") is None or kwargs.get("v_scale_cache") is None))
        or (descaled and mode != KVQuantMode.FP8_PER_TENSOR)
        or kwargs.get("alibi_slopes") is not None
        or kwargs.get("sinks") is not None
        or kwargs.get("softcap", 0.0) != 0.0
        or tuple(kwargs.get("window_size", (-1, -1))) != (-1, -1)
        or kwargs.get("q_descale") is not None
        or kwargs.get("use_td", False)
        or kwargs.get("causal") is not True
        or not kernel_supports(kwargs["q"], kwargs["k"], int(mode))
    )
    decode_only = max_query_len <= 1
    if not enabled or unsupported or max_query_len < 1 or (decode_only and not _flag("ILUVATAR_SPLIT_KV_DECODE")):
        return _vllm_unified_attention()(**kwargs)
    num_splits = int(os.environ.get("ILUVATAR_NUM_SPLITS", "0") or 0)
    return unified_attention_optimized(
        q=kwargs["q"],
        k=kwargs["k"],
        v=kwargs["v"],
        out=kwargs["out"],
        block_table=kwargs["block_table"],
        seqused_k=kwargs["seqused_k"],
        cu_seqlens_q=kwargs["cu_seqlens_q"],
        max_seqlen_q=kwargs["max_seqlen_q"],
        max_seqlen_k=kwargs["max_seqlen_k"],
        softmax_scale=kwargs["softmax_scale"],
        causal=kwargs["causal"],
        num_splits_override=num_splits or None,
        block_m_override=int(os.environ.get("ILUVATAR_BLOCK_M", "64")),
        block_n_override=int(os.environ.get("ILUVATAR_BLOCK_N", "64")),
        launch_num_warps_override=int(os.environ.get("ILUVATAR_NUM_WARPS", "4")),
        launch_num_stages_override=int(os.environ.get("ILUVATAR_NUM_STAGES", "2")),
        kv_quant_mode=int(mode),
        k_descale=kwargs.get("k_descale"),
        v_descale=kwargs.get("v_descale"),
        k_scale_cache=kwargs.get("k_scale_cache"),
        v_scale_cache=kwargs.get("v_scale_cache"),
    )


@dataclass
class IluvatarAttentionMetadata:
    """Per-step attention metadata (fields of the reference's dataclass, patch :150-187)."""

    num_actual_tokens: int
    max_query_len: int
    query_start_loc: torch.Tensor
    max_seq_len: int
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    slot_mapping: torch.Tensor

    seq_threshold_3D: int
    num_par_softmax_segments: int
    softmax_segm_output: torch.Tensor
    softmax_segm_max: torch.Tensor
    softmax_segm_expsum: torch.Tensor

    causal: bool | torch.Tensor

    use_cascade: bool
    common_prefix_len: int
    cu_prefix_query_lens: torch.Tensor | None
    prefix_kv_lens: torch.Tensor | None
    suffix_kv_lens: torch.Tensor | None

    scheduler_metadata: torch.Tensor | None = None
    prefix_scheduler_metadata: torch.Tensor | None = None
    mm_prefix_range: dict[int, list[tuple[int, int]]] | None = None
    mm_prefix_range_tensor: torch.Tensor | None = None


def _next_power_of_2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


class IluvatarAttentionMetadataBuilder:
    """Builds :class:`IluvatarAttentionMetadata` from the scheduler's common metadata (patch :189-336).

    ``common`` is any object with the fields of vLLM's
    ``CommonAttentionMetadata`` that the reference reads: ``num_reqs``,
    ``num_actual_tokens``, ``max_query_len``, ``max_seq_len``,
    ``query_start_loc``, ``seq_lens``, ``block_table_tensor``,
    ``slot_mapping``, ``causal`` (and optionally ``mm_req_doc_ranges``).
    The 3D-softmax scratch is allocated as in the reference; only vLLM's
    baseline kernel uses it.
    """

    def __init__(self, num_heads_q: int, num_heads_kv: int, head_dim: int, device: torch.device,
                 cudagraph_capture_sizes: list[int] | None = None):
        self.num_heads_q = num_heads_q
        self.num_heads_kv = num_heads_kv
        self.headdim = head_dim
        self.device = torch.device(device)
        self.seq_threshold_3D = MIN_LAUNCH_GRID_SIZE_2D // num_heads_kv
        if cudagraph_capture_sizes:
            self.seq_threshold_3D = min(cudagraph_capture_sizes, key=lambda x: abs(x - self.seq_threshold_3D))
        self.num_par_softmax_segments = NUM_PAR_SOFTMAX_SEGMENTS
        padded = _next_power_of_2(head_dim)
        shape = (self.seq_threshold_3D, num_heads_q, self.num_par_softmax_segments)
        self.softmax_segm_output = torch.empty(shape + (padded,), dtype=torch.float32, device=self.device)
        self.softmax_segm_max = torch.empty(shape, dtype=torch.float32, device=self.device)
        self.softmax_segm_expsum = torch.empty(shape, dtype=torch.float32, device=self.device)

    def build(self, common_prefix_len: int, common: Any, fast_build: bool = False) -> IluvatarAttentionMetadata:
        use_cascade = common_prefix_len > 0
        if use_cascade:
            cu_prefix = torch.tensor([0, common.num_actual_tokens], dtype=torch.int32, device=self.device)
            prefix_kv = torch.tensor([common_prefix_len], dtype=torch.int32, device=self.device)
            suffix_kv = (common.seq_lens.cpu() - common_prefix_len).to(self.device)
        else:
            cu_prefix = prefix_kv = suffix_kv = None
        meta = IluvatarAttentionMetadata(
            num_actual_tokens=common.num_actual_tokens,
            max_query_len=common.max_query_len,
            query_start_loc=common.query_start_loc,
            max_seq_len=common.max_seq_len,
            seq_lens=common.seq_lens,
            block_table=common.block_table_tensor,
            slot_mapping=common.slot_mapping,
            causal=common.causal,
            use_cascade=use_cascade,
            common_prefix_len=common_prefix_len,
            cu_prefix_query_lens=cu_prefix,
            prefix_kv_lens=prefix_kv,
            suffix_kv_lens=suffix_kv,
            seq_threshold_3D=self.seq_threshold_3D,
            num_par_softmax_segments=self.num_par_softmax_segments,
            softmax_segm_output=self.softmax_segm_output,
            softmax_segm_max=self.softmax_segm_max,
            softmax_segm_expsum=self.softmax_segm_expsum,
        )
        ranges = getattr(common, "mm_req_doc_ranges", None)
        if ranges is not None:
            meta.mm_prefix_range = ranges
        return meta

    def build_for_cudagraph_capture(self, common: Any) -> IluvatarAttentionMetadata:
        meta = self.build(0, common)
        meta.seq_lens.fill_(1)  # as the reference: keeps graph capture fast
        return meta


class IluvatarAttentionBackend:
    """The backend's static contract (patch :339-466)."""

    supported_dtypes: ClassVar[list[torch.dtype]] = [torch.float16, torch.bfloat16, torch.float32]
    supported_kv_cache_dtypes: ClassVar[list[str]] = [
        "auto", "float16", "bfloat16", "fp8", "fp8_e4m3", "fp8_e5m2", "int8_per_token_head", "fp8_per_token_head",
    ]
    forward_includes_kv_cache_update: bool = False

    @staticmethod
    def get_name() -> str:
        return "TRITON_ATTN"

    @staticmethod
    def get_impl_cls() -> type["IluvatarAttentionImpl"]:
        return IluvatarAttentionImpl

    @staticmethod
    def get_builder_cls() -> type[IluvatarAttentionMetadataBuilder]:
        return IluvatarAttentionMetadataBuilder

    @staticmethod
    def get_supported_kernel_block_sizes() -> list[str]:
        return ["multiple of 16"]

    @classmethod
    def supports_block_size(cls, block_size: int | None) -> bool:
        return block_size is None or block_size % 16 == 0

    @classmethod
    def supports_non_causal(cls) -> bool:
        return True

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size >= 32

    @classmethod
    def supports_attn_type(cls, attn_type: str) -> bool:
        return attn_type in (AttentionType.DECODER, AttentionType.ENCODER, AttentionType.ENCODER_ONLY,
                             AttentionType.ENCODER_DECODER)

    @staticmethod
    def use_cascade_attention(*args, **kwargs) -> bool:
        return False

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        if block_size % 16 != 0:
            raise ValueError("Block size must be a multiple of 16.")
        if get_kv_quant_mode(cache_dtype_str).is_per_token_head:
            # One float32 scale inline after head_size (4 one-byte elements).
            return (num_blocks, 2, block_size, num_kv_heads, head_size + 4)
        return (num_blocks, 2, block_size, num_kv_heads, head_size)

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension: bool = False, cache_layout: str = "NHD") -> tuple[int, ...]:
        if cache_layout == "NHD":
            return (1, 0, 2, 3, 4, 5) if include_num_layers_dimension else (0, 1, 2, 3, 4)
        if cache_layout == "HND":
            return (1, 4, 0, 2, 3, 5) if include_num_layers_dimension else (0, 1, 3, 2, 4)
        raise ValueError(f"Unknown cache layout: {cache_layout}")


class IluvatarAttentionImpl:
    """Attention layer implementation of the service (patch :468-899), on the sm_100a operators."""

    _k_scale_cache: torch.Tensor | None = None
    _v_scale_cache: torch.Tensor | None = None

    def __init__(
        self,
        num_heads: int,
        head_size: int,
        scale: float,
        num_kv_heads: int,
        alibi_slopes: list[float] | None,
        sliding_window: int | None,
        kv_cache_dtype: str,
        logits_soft_cap: float | None = None,
        attn_type: str = AttentionType.DECODER,
        kv_sharing_target_layer_name: str | None = None,
        sinks: torch.Tensor | None = None,
        use_alibi_sqrt: bool = False,
        chunk_lookback: int = -1,
    ) -> None:
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = float(scale)
        self.num_kv_heads = num_kv_heads
        self.alibi_slopes = torch.tensor(alibi_slopes, dtype=torch.float32) if alibi_slopes is not None else None
        if sliding_window is None:
            self.sliding_window = (-1, -1)
        elif attn_type in (AttentionType.ENCODER, AttentionType.ENCODER_ONLY):
            self.sliding_window = (sliding_window - 1, sliding_window - 1)
        else:
            self.sliding_window = (sliding_window - 1, 0)
        self.kv_cache_dtype = kv_cache_dtype
        self.logits_soft_cap = 0 if logits_soft_cap is None else logits_soft_cap
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        self.num_queries_per_kv = num_heads // num_kv_heads
        self.attn_type = attn_type
        self.fp8_dtype = FP8_DTYPE
        self.sinks = sinks
        if sinks is not None and sinks.shape[0] != num_heads:
            raise AssertionError(
                "Sinks must have the same number of heads as the number of heads in the layer. "
                f"Sinks shape: {sinks.shape}, num_heads: {num_heads}."
            )
        self.use_alibi_sqrt = use_alibi_sqrt
        self.chunk_lookback = chunk_lookback
        self._kv_quant_mode = get_kv_quant_mode(kv_cache_dtype)
        self._is_per_token_head_quant = self._kv_quant_mode.is_per_token_head
        self.use_td = False  # tensor descriptors: an Intel Xe option of vLLM's kernel

    # ------------------------------------------------------------------ caches
    def _ensure_scale_caches(self, kv_cache: torch.Tensor) -> None:
        """float32 views of the per-(block, slot, head) scales stored after head_size (patch :473-523)."""
        if self._k_scale_cache is not None:
            return
        num_blocks, _, block_size, nkv, padded = kv_cache.shape
        e = kv_cache.element_size()
        pad = 4 // e
        hs = padded - pad
        base = torch.empty(0, dtype=torch.float32, device=kv_cache.device).set_(kv_cache.untyped_storage())
        half = block_size * nkv * padded * e
        stride = (2 * half // 4, nkv * padded * e // 4, padded * e // 4)
        start = kv_cache.storage_offset() * e // 4 + hs * e // 4
        self._k_scale_cache = torch.as_strided(base, (num_blocks, block_size, nkv), stride, start)
        self._k_scale_cache.fill_(1.0)
        self._v_scale_cache = torch.as_strided(base, (num_blocks, block_size, nkv), stride, start + half // 4)
        self._v_scale_cache.fill_(1.0)

    def _split_cache(self, kv_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """``kv_cache.unbind(1)``, viewed as fp8 where the reference views it (per-token-head rows keep their padding)."""
        key_cache, value_cache = kv_cache.unbind(1)
        if self._is_per_token_head_quant:
            if key_cache.dtype == torch.uint8:
                key_cache, value_cache = key_cache.view(self.fp8_dtype), value_cache.view(self.fp8_dtype)
        elif is_quantized_kv_cache(self.kv_cache_dtype) and key_cache.dtype != self.fp8_dtype:
            key_cache, value_cache = key_cache.view(self.fp8_dtype), value_cache.view(self.fp8_dtype)
        return key_cache, value_cache

    def fused_output_quant_supported(self, quant_key: Any) -> bool:
        return False

    # ------------------------------------------------------------------ forward
    def forward(
        self,
        layer: Any,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        kv_cache: torch.Tensor,
        attn_metadata: IluvatarAttentionMetadata | None,
        output: torch.Tensor,
        output_scale: torch.Tensor | None = None,
        output_block_scale: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Paged attention of ``query [T, H, D]`` over ``kv_cache [blocks, 2, bs, KH, D]`` into ``output``."""
        if output_block_scale is not None:
            raise NotImplementedError(
                "fused block_scale output quantization is not yet supported for IluvatarAttentionImpl"
            )
        if attn_metadata is None:  # profiling run
            return output.fill_(0)
        assert attn_metadata.use_cascade is False
        n = attn_metadata.num_actual_tokens
        if self.attn_type in (AttentionType.ENCODER_ONLY, AttentionType.ENCODER):
            return self._forward_encoder_attention(query[:n], key[:n], value[:n], output[:n], attn_metadata, layer)

        if self._is_per_token_head_quant:
            self._ensure_scale_caches(kv_cache)
            key_cache, value_cache = self._split_cache(kv_cache)
            q_descale = k_descale = v_descale = None
            k_scale_cache, v_scale_cache = self._k_scale_cache, self._v_scale_cache
        else:
            key_cache, value_cache = self._split_cache(kv_cache)
            quantized = self._kv_quant_mode == KVQuantMode.FP8_PER_TENSOR
            descale_shape = (attn_metadata.query_start_loc.shape[0] - 1, key_cache.shape[2])
            q_descale = layer._q_scale if (quantized and query.dtype == self.fp8_dtype) else None
            # Descales only for a quantised cache (the reference passed them for
            # every cache, which kept the service off the optimized path).
            k_descale = layer._k_scale.expand(descale_shape) if quantized else None
            v_descale = layer._v_scale.expand(descale_shape) if quantized else None
            k_scale_cache = v_scale_cache = None

        _run_unified_attention(
            q=query[:n],
            k=key_cache,
            v=value_cache,
            out=output[:n],
            cu_seqlens_q=attn_metadata.query_start_loc,
            max_seqlen_q=attn_metadata.max_query_len,
            seqused_k=attn_metadata.seq_lens,
            max_seqlen_k=attn_metadata.max_seq_len,
            softmax_scale=self.scale,
            causal=attn_metadata.causal,
            alibi_slopes=self.alibi_slopes,
            use_alibi_sqrt=self.use_alibi_sqrt,
            window_size=self.sliding_window,
            block_table=attn_metadata.block_table,
            softcap=self.logits_soft_cap,
            q_descale=q_descale,
            k_descale=k_descale,
            v_descale=v_descale,
            seq_threshold_3D=attn_metadata.seq_threshold_3D,
            num_par_softmax_segments=attn_metadata.num_par_softmax_segments,
            softmax_segm_output=attn_metadata.softmax_segm_output,
            softmax_segm_max=attn_metadata.softmax_segm_max,
            softmax_segm_expsum=attn_metadata.softmax_segm_expsum,
            sinks=self.sinks,
            output_scale=output_scale,
            mm_prefix_range=attn_metadata.mm_prefix_range_tensor,
            kv_quant_mode=self._kv_quant_mode,
            k_scale_cache=k_scale_cache,
            v_scale_cache=v_scale_cache,
            chunk_lookback=self.chunk_lookback,
            use_td=self.use_td,
        )
        return output

    def _forward_encoder_attention(self, query, key, value, output, attn_metadata, layer) -> torch.Tensor:
        """Bidirectional attention without a cache: vLLM's ``context_attention_fwd``, as in the reference."""
        if is_quantized_kv_cache(self.kv_cache_dtype):
            raise NotImplementedError("quantized KV cache is not supported for encoder attention")
        try:
            from vllm.v1.attention.ops.triton_prefill_attention import context_attention_fwd
        except Exception as exc:
            raise RuntimeError(f"encoder attention stays on vLLM's context_attention_fwd, which is unavailable: {exc}") from exc
        context_attention_fwd(
            q=query, k=key, v=value, o=output, b_start_loc=attn_metadata.query_start_loc,
            b_seq_len=attn_metadata.seq_lens, max_input_len=attn_metadata.max_query_len, is_causal=False,
            softmax_scale=self.scale, sliding_window_q=self.sliding_window[0], sliding_window_k=self.sliding_window[1],
        )
        return output

    # ------------------------------------------------------------------ cache updates
    def do_kv_cache_update(self, layer: Any, key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
                           slot_mapping: torch.Tensor) -> None:
        """Write the step's new K/V rows into the paged cache (patch :815-858)."""
        if self.attn_type in (AttentionType.ENCODER_ONLY, AttentionType.ENCODER):
            return
        if self._is_per_token_head_quant:
            self._ensure_scale_caches(kv_cache)
            key_cache, value_cache = self._split_cache(kv_cache)
            reshape_and_cache_flash_per_token_head_quant(
                key, value, key_cache, value_cache, self._k_scale_cache, self._v_scale_cache, slot_mapping
            )
            return
        key_cache, value_cache = self._split_cache(kv_cache)
        reshape_and_cache_flash(key, value, key_cache, value_cache, slot_mapping, self.kv_cache_dtype,
                                layer._k_scale, layer._v_scale)

    def fused_rope_kvcache_supported(self) -> bool:
        return not self._is_per_token_head_quant

    def do_rope_and_kv_cache_update(self, layer: Any, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                    positions: torch.Tensor, cos_sin_cache: torch.Tensor, is_neox: bool,
                                    kv_cache: torch.Tensor, layer_slot_mapping: torch.Tensor) -> None:
        """Rotate query and key in place and write the rotated key and the value to the cache (patch :865-899)."""
        key_cache, value_cache = kv_cache.unbind(1)
        is_fp8 = is_quantized_kv_cache(self.kv_cache_dtype)
        if is_fp8:
            key_cache, value_cache = key_cache.view(self.fp8_dtype), value_cache.view(self.fp8_dtype)
        rope_and_cache(query, key, value, positions, cos_sin_cache, is_neox, key_cache, value_cache,
                       layer_slot_mapping, layer._k_scale, layer._v_scale, True, is_fp8)


__all__ = [
    "KVQuantMode",
    "get_kv_quant_mode",
    "AttentionType",
    "IluvatarAttentionMetadata",
    "IluvatarAttentionMetadataBuilder",
    "IluvatarAttentionBackend",
    "IluvatarAttentionImpl",
    "_run_unified_attention",
]
