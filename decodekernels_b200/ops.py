"""Python wrapper of ``torch.ops.decode_kernels.paged_attention_decode``.

Same public surface as DecodeKernels' ``decode_kernels/ops.py:14-116`` for the
attention path: ``PARTITION_SIZE``, ``MAX_GQA_GROUP``, ``SUPPORTED_HEAD_DIMS``,
``is_available``, ``num_partitions``, ``alloc_workspace`` and
``paged_attention_decode`` with the same signature, defaults and errors.  The
op is mutating (``Tensor!`` arguments), so it can run on preallocated buffers
inside CUDA graphs.

Differences that stay within the reference's contract:

* ``alloc_workspace`` sizes the split-K workspace for this library's per-shape
  planner (partitions of 512 KB to 2 MB of K+V -- 1024 to 4096 tokens at
  head_dim 128 with 16-bit caches -- chosen to fill all SMs), and never
  smaller than the reference's ``ceil(max_seq_len / 512)`` partitions.  Optional
  keyword ``num_kv_heads`` sizes it exactly; without it the size covers any
  head count.
* A non-empty workspace is also used when ``max_seq_len <= 512`` (small
  batches split to fill the GPU).
* A 4-tuple workspace ``(tmp_out, max_logits, exp_sums, merge_counters)``
  (``alloc_workspace(..., merge_counters=True)``) goes through
  ``decode_kernels::paged_attention_decode_fused``, which may merge the
  partitions inside the partition kernel (one launch instead of two).

The native library is loaded from ``decodekernels_b200/lib``.  If it is not
built, ``is_available()`` is False and every op raises; there is no CPU
fallback.
"""

from __future__ import annotations

import math
from pathlib import Path

import torch

from . import capi

PARTITION_SIZE = 512  # the reference's split-K partition; the workspace is never smaller than its ceil(L / 512)
MAX_GQA_GROUP = capi.DK_MAX_GQA_GROUP
SUPPORTED_HEAD_DIMS = (64, 128, 256)
FLAG_PERSISTENT = capi.DK_FLAG_PERSISTENT  # one wave of CTAs over the live work items

TORCH_LIB_PATH = Path(__file__).resolve().parent / "lib" / "libdk_b200_torch.so"

def _register_fakes() -> None:
    """Fake (meta) implementations let torch.compile trace through the ops."""

    @torch.library.register_fake("decode_kernels::paged_attention_decode")
    def _(out, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums):
        return None

    @torch.library.register_fake("decode_kernels::paged_attention_decode_fused")
    def _(out, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums,
          merge_counters):
        return None

    @torch.library.register_fake("decode_kernels::reshape_and_cache")
    def _(key, value, key_cache, value_cache, slot_mapping, k_scale, v_scale):
        return None

    @torch.library.register_fake("decode_kernels::paged_attention_decode_lse")
    def _(partial, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums,
          k_scale=1.0, v_scale=1.0):
        return None

    @torch.library.register_fake("decode_kernels::paged_attention_decode_ext")
    def _(out, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums,
          merge_counters, k_scale, v_scale, flags=0):
        return None

    @torch.library.register_fake("decode_kernels::merge_lse")
    def _(out, parts):
        return None


_AVAILABLE = False
_IMPORT_ERROR: Exception | None = None


def load_native() -> bool:
    """Load both native libraries (at import, and again after a build in
    the same process); True when they are loaded.  A missing or stale library
    leaves every op raising -- nothing falls back."""
    global _AVAILABLE, _IMPORT_ERROR
    if _AVAILABLE:
        return True
    try:
        if not TORCH_LIB_PATH.exists():
            raise ImportError(f"{TORCH_LIB_PATH} is not built")
        torch.ops.load_library(str(TORCH_LIB_PATH))  # registers torch.ops.decode_kernels.*
        capi._lib = None  # a failed earlier load must not stick
        capi.load()
        _register_fakes()
        _AVAILABLE, _IMPORT_ERROR = True, None
    except Exception as e:
        _AVAILABLE, _IMPORT_ERROR = False, e
    return _AVAILABLE


load_native()


def is_available() -> bool:
    """True when the native library is built and a GPU is visible."""
    return _AVAILABLE and torch.cuda.is_available()


def _require() -> None:
    if not _AVAILABLE:
        raise RuntimeError(
            "decodekernels_b200 native library is not built. Run `python -m decodekernels_b200.build` on a "
            f"machine with nvcc. Original error: {_IMPORT_ERROR}"
        )


def num_partitions(max_seq_len: int) -> int:
    """Partitions of the reference's fixed 512-token split (ops.py:67-68)."""
    return max(1, math.ceil(max_seq_len / PARTITION_SIZE))


def _device_index(device) -> int:
    d = torch.device(device)
    if d.type != "cuda":
        return -1
    return d.index if d.index is not None else (torch.cuda.current_device() if torch.cuda.is_available() else -1)


def alloc_workspace(num_seqs: int, num_q_heads: int, head_dim: int, max_seq_len: int, device, *,
                    num_kv_heads: int | None = None, block_size: int = 16, merge_counters: bool = False) -> tuple:
    """Split-K buffers ``(tmp_out, max_logits, exp_sums)`` for a call with these
    sizes, or three empty tensors when the call will run single-pass.

    Shapes: ``tmp_out [num_seqs, num_q_heads, P, head_dim]``, the other two
    ``[num_seqs, num_q_heads, P]``, float32, with ``P`` the planner's partition
    count (at least the reference's ``ceil(max_seq_len / 512)``).

    ``merge_counters=True`` (needs ``num_kv_heads``) appends a zeroed int32
    ``[num_seqs * num_kv_heads]`` tensor: calls given this 4-tuple merge the
    partitions inside the partition kernel (one launch instead of two).  The
    counters return to zero after every completed call; calls that may run
    concurrently need separate workspaces.
    """
    _require()
    try:
        parts = capi.num_partitions(num_seqs, num_kv_heads or 0, head_dim, block_size, max_seq_len,
                                    _device_index(device))
    except ValueError:
        parts = 1  # unsupported shape: size like the reference and let the op report the error
    parts = max(parts, num_partitions(max_seq_len))
    if parts <= 1 and max_seq_len <= PARTITION_SIZE:
        empty = torch.empty(0, dtype=torch.float32, device=device)
        return empty, empty, empty
    tmp_out = torch.empty(num_seqs, num_q_heads, parts, head_dim, dtype=torch.float32, device=device)
    max_logits = torch.empty(num_seqs, num_q_heads, parts, dtype=torch.float32, device=device)
    exp_sums = torch.empty_like(max_logits)
    if merge_counters:
        if not num_kv_heads:
            raise ValueError("merge_counters=True needs num_kv_heads")
        return tmp_out, max_logits, exp_sums, torch.zeros(num_seqs * num_kv_heads, dtype=torch.int32, device=device)
    return tmp_out, max_logits, exp_sums


def paged_attention_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    max_seq_len: int | None = None,
    out: torch.Tensor | None = None,
    workspace: tuple | None = None,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
    flags: int = 0,
) -> torch.Tensor:
    """Single-token decode attention over a paged KV cache.

    q: [num_seqs, num_q_heads, head_dim]; k_cache / v_cache:
    [num_blocks, block_size, num_kv_heads, head_dim] (any strides on the first
    three dims); block_tables: [num_seqs, max_blocks] int32; seq_lens:
    [num_seqs] int32. ``max_seq_len`` must be >= every entry of seq_lens; pass
    it when known to avoid a device-to-host sync.

    Caches of dtype uint8 / float8_e4m3fn hold e4m3 codes (as written by
    :func:`reshape_and_cache`): K = code * k_scale, V = code * v_scale.
    ``flags``: ``DK_FLAG_*`` bits of the C ABI (``capi.DK_FLAG_PERSISTENT``:
    one wave of CTAs over the live work items, for a grid planned from a
    large ``max_seq_len`` such as a CUDA graph captured for a model's
    maximum length).
    """
    _require()
    num_seqs, num_q_heads, head_dim = q.shape
    if scale is None:
        scale = head_dim**-0.5
    if max_seq_len is None:
        max_seq_len = int(seq_lens[:num_seqs].max().item()) if num_seqs > 0 else 0
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        kv_heads = k_cache.shape[2] if k_cache.dim() == 4 else None
        bs = k_cache.shape[1] if k_cache.dim() == 4 else 16
        workspace = alloc_workspace(num_seqs, num_q_heads, head_dim, max_seq_len, q.device, num_kv_heads=kv_heads,
                                    block_size=bs)
    tmp_out, max_logits, exp_sums = workspace[:3]
    counters = workspace[3] if len(workspace) > 3 else None
    if flags or k_cache.dtype in (torch.uint8, torch.float8_e4m3fn):
        torch.ops.decode_kernels.paged_attention_decode_ext(
            out, q, k_cache, v_cache, block_tables, seq_lens, float(scale), int(max_seq_len), tmp_out, max_logits,
            exp_sums, counters, float(k_scale), float(v_scale), int(flags)
        )
    elif counters is not None:
        torch.ops.decode_kernels.paged_attention_decode_fused(
            out, q, k_cache, v_cache, block_tables, seq_lens, float(scale), int(max_seq_len), tmp_out, max_logits,
            exp_sums, counters
        )
    else:
        torch.ops.decode_kernels.paged_attention_decode(
            out, q, k_cache, v_cache, block_tables, seq_lens, float(scale), int(max_seq_len), tmp_out, max_logits,
            exp_sums
        )
    return out


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                      slot_mapping: torch.Tensor, k_scale: float = 1.0, v_scale: float = 1.0) -> None:
    """Paged-KV write, the step before decode (vLLM's ``reshape_and_cache_flash``).

    key / value: [num_tokens, num_kv_heads, head_dim] (fp16/bf16);
    key_cache / value_cache: [num_blocks, block_size, num_kv_heads, head_dim]
    in any of the decode's layouts, with key's dtype or uint8 /
    float8_e4m3fn (stored as ``sat_e4m3(x / scale)``); slot_mapping: int64
    [num_tokens], ``block * block_size + offset``, negative = padding.
    """
    _require()
    torch.ops.decode_kernels.reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, float(k_scale),
                                               float(v_scale))


def paged_attention_decode_lse(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    max_seq_len: int | None = None,
    partial: torch.Tensor | None = None,
    workspace: tuple | None = None,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    """Decode attention as fp32 partials: ``[num_seqs, num_q_heads, head_dim + 4]``
    rows holding the normalised output ``o``, then ``lse = log(sum_t exp(scale * q.k_t))``
    (``-inf`` and ``o = 0`` for an empty sequence), then 3 unused floats.

    Partials of disjoint token ranges of the same sequences (the shards of a
    sequence-sharded cache) combine exactly with :func:`merge_lse`.  Arguments
    are as in :func:`paged_attention_decode`.
    """
    _require()
    num_seqs, num_q_heads, head_dim = q.shape
    if scale is None:
        scale = head_dim**-0.5
    if max_seq_len is None:
        max_seq_len = int(seq_lens[:num_seqs].max().item()) if num_seqs > 0 else 0
    if partial is None:
        partial = torch.empty(num_seqs, num_q_heads, head_dim + 4, dtype=torch.float32, device=q.device)
    if workspace is None:
        kv_heads = k_cache.shape[2] if k_cache.dim() == 4 else None
        bs = k_cache.shape[1] if k_cache.dim() == 4 else 16
        workspace = alloc_workspace(num_seqs, num_q_heads, head_dim, max_seq_len, q.device, num_kv_heads=kv_heads,
                                    block_size=bs)
    tmp_out, max_logits, exp_sums = workspace[:3]
    torch.ops.decode_kernels.paged_attention_decode_lse(partial, q, k_cache, v_cache, block_tables, seq_lens,
                                                        float(scale), int(max_seq_len), tmp_out, max_logits,
                                                        exp_sums, float(k_scale), float(v_scale))
    return partial


def merge_lse(parts: torch.Tensor, out: torch.Tensor | None = None, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Combine partials of disjoint token ranges, ``parts [R, n, Hq, D + 4]``
    (from :func:`paged_attention_decode_lse`), into the attention output
    ``[n, Hq, D]`` of ``out``'s dtype (``dtype`` when ``out`` is None), or into
    merged fp32 partial rows when ``out`` is float32 ``[n, Hq, D + 4]``."""
    _require()
    if out is None:
        out = torch.empty(parts.shape[1], parts.shape[2], parts.shape[3] - 4, dtype=dtype, device=parts.device)
    torch.ops.decode_kernels.merge_lse(out, parts)
    return out
