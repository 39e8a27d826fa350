"""Swap this library's paged-attention decode into vLLM.

The same surface as DecodeKernels' ``decode_kernels/vllm_patch.py`` (``apply``,
``stats``, ``reset_stats``; ``decode_kernels/vllm_patch.py:47-55,200-211``),
re-targeted at the vLLM installed here (0.22, v1 engine, FlashAttention
backend):

* ``FlashAttentionImpl.forward`` -- pure-decode batches (one query token per
  request) run ``paged_attention_decode`` on vLLM's KV cache in place.  vLLM
  0.22 stores the cache as ``[2, num_blocks, block_size, num_kv_heads,
  head_size]`` (any stride order) and splits it with ``kv_cache.unbind(0)``;
  the kernel reads those two strided views directly.  The reference's patch
  built its views with ``kv_cache.transpose(1, 2).split(head_size, -1)``
  for an older interleaved layout (``decode_kernels/vllm_patch.py:122``).
  vLLM writes the new token's K/V before ``forward`` runs, so ``seq_lens``
  already includes it.
* FP8 KV caches (``kv_cache_dtype`` "fp8" / "fp8_e4m3": uint8 e4m3 codes
  written with the layer's per-tensor scales) decode here too, with
  ``layer._k_scale_float`` / ``layer._v_scale_float``, as long as the query
  stays 16-bit.  The reference refuses every quantized cache
  (``decode_kernels/vllm_patch.py:74``); this library has an e4m3 path.
* CUDA-graph capture (vLLM's full-cudagraph mode) is served too, where the
  reference refused it (``decode_kernels/vllm_patch.py:65-69``): vLLM builds
  the metadata it captures with ``max_seq_len = max_model_len``
  (``v1/worker/gpu_model_runner.py``, ``for_cudagraph_capture``), a bound on
  every replay's lengths, and refreshes ``seq_lens`` and ``block_table`` in
  place before each replay, which the kernels read on the device.  A grid
  planned for the model's maximum length is mostly empty at replay, so a
  captured call takes the persistent grid (``FLAG_PERSISTENT``: one wave of
  CTAs over the live work items).
* Everything else falls back to the original FlashAttention path through a
  strict eligibility check (``_attention_eligible``): prefill and mixed
  batches, e5m2 or other quantized caches, fp8 queries, sliding windows,
  ALiBi, soft-capping, sinks, cascade attention, context parallelism,
  head sizes other than 64/128/256 and GQA groups above 8.
* ``rms_norm`` and ``silu_and_mul`` (the reference's other two patches) are
  not part of this library; asking for them logs a note and changes nothing.
"""

from __future__ import annotations

import logging

import torch

from . import ops as dk_ops

logger = logging.getLogger("decodekernels_b200.vllm")

_STATS = {"attention_kernel_calls": 0, "attention_fallback_calls": 0}
_APPLIED: set[str] = set()
_HALF_TYPES = (torch.float16, torch.bfloat16)
_NOT_PROVIDED = ("rms_norm", "silu_and_mul")


def stats() -> dict[str, int]:
    """How often the patched attention used this library vs fell back."""
    return dict(_STATS)


def reset_stats() -> None:
    for k in _STATS:
        _STATS[k] = 0


_FP8_E4M3 = ("fp8", "fp8_e4m3")


def _fp8_scales(layer) -> tuple[float, float] | None:
    """The layer's per-tensor K/V scales as floats, or None when unusable."""
    ks, vs = getattr(layer, "_k_scale_float", None), getattr(layer, "_v_scale_float", None)
    try:
        ks, vs = float(ks), float(vs)
    except (TypeError, ValueError):
        return None
    if not (0.0 < ks < float("inf") and 0.0 < vs < float("inf")):
        return None
    return ks, vs


def _attention_eligible(impl, query, kv_cache, attn_metadata, output, output_scale, output_block_scale,
                        layer=None) -> bool:
    """True when this decode batch can run on decodekernels_b200 unchanged."""
    if attn_metadata is None or output_scale is not None or output_block_scale is not None:
        return False
    try:
        from vllm.v1.attention.backend import AttentionType

        decoder = AttentionType.DECODER
    except ImportError:  # pragma: no cover - depends on the vLLM build
        decoder = "decoder"
    if getattr(impl, "attn_type", decoder) != decoder or getattr(attn_metadata, "max_query_len", None) != 1:
        return False
    if getattr(attn_metadata, "use_cascade", False):
        return False
    if getattr(impl, "dcp_world_size", 1) > 1:
        return False
    kv_dtype = str(getattr(impl, "kv_cache_dtype", "auto"))
    if query.dtype not in _HALF_TYPES:
        return False
    if kv_dtype in ("auto", "float16", "bfloat16"):
        if kv_cache.dtype != query.dtype:
            return False
    elif kv_dtype in _FP8_E4M3:
        if kv_cache.dtype not in (torch.uint8, torch.float8_e4m3fn) or _fp8_scales(layer) is None:
            return False
    else:
        return False
    if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
        return False
    if getattr(impl, "alibi_slopes", None) is not None or getattr(impl, "logits_soft_cap", None):
        return False
    if getattr(impl, "sliding_window", None) not in (None, (-1, -1)):
        return False
    if getattr(impl, "sinks", None) is not None:
        return False
    if impl.head_size not in dk_ops.SUPPORTED_HEAD_DIMS:
        return False
    if impl.num_heads % impl.num_kv_heads or impl.num_heads // impl.num_kv_heads > dk_ops.MAX_GQA_GROUP:
        return False
    if getattr(attn_metadata, "causal", True) is not True:
        return False
    n = attn_metadata.num_actual_tokens
    if attn_metadata.seq_lens.shape[0] < n or attn_metadata.block_table.shape[0] < n:
        return False
    if not output.is_contiguous():
        return False
    return True


def _decode(impl, query, kv_cache, attn_metadata, output, layer=None) -> torch.Tensor:
    n = attn_metadata.num_actual_tokens
    key_cache, value_cache = kv_cache.unbind(0)  # two [blocks, bs, heads, D] views, read in place
    q = query[:n].reshape(n, impl.num_heads, impl.head_size)
    out = output[:n].view(n, impl.num_heads, impl.head_size)
    k_scale, v_scale = 1.0, 1.0
    if str(getattr(impl, "kv_cache_dtype", "auto")) in _FP8_E4M3:
        k_scale, v_scale = _fp8_scales(layer)
    # Under capture the grid is planned from max_seq_len (vLLM passes the
    # model's maximum length) and replayed with other lengths: persistent grid.
    flags = dk_ops.FLAG_PERSISTENT if query.is_cuda and torch.cuda.is_current_stream_capturing() else 0
    dk_ops.paged_attention_decode(q, key_cache, value_cache, attn_metadata.block_table, attn_metadata.seq_lens,
                                  scale=impl.scale, max_seq_len=attn_metadata.max_seq_len, out=out, k_scale=k_scale,
                                  v_scale=v_scale, flags=flags)
    return output


def _patch_attention() -> None:
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl

    original = FlashAttentionImpl.forward

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if _attention_eligible(self, query, kv_cache, attn_metadata, output, output_scale, output_block_scale, layer):
            _STATS["attention_kernel_calls"] += 1
            return _decode(self, query, kv_cache, attn_metadata, output, layer)
        _STATS["attention_fallback_calls"] += 1
        return original(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                        output_block_scale)

    forward.__wrapped__ = original  # type: ignore[attr-defined]
    FlashAttentionImpl.forward = forward


_PATCHERS = {"attention": _patch_attention}


def apply(ops: list[str] | None = None) -> None:
    """Install the patches (idempotent)."""
    if not dk_ops.is_available():
        logger.warning("decodekernels_b200: native library or GPU unavailable; vLLM left unpatched")
        return
    for name in ops or list(_PATCHERS):
        if name in _NOT_PROVIDED:
            logger.info("decodekernels_b200 provides no %s kernel; vLLM keeps its own", name)
            continue
        if name not in _PATCHERS:
            raise ValueError(f"unknown op {name!r}; choose from {sorted(_PATCHERS)}")
        if name in _APPLIED:
            continue
        _PATCHERS[name]()
        _APPLIED.add(name)
    logger.info("decodekernels_b200: patched vLLM ops %s", sorted(_APPLIED))
