"""CPU oracle for paged-attention decode.  TEST INFRASTRUCTURE, NOT PRODUCT.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this module, and only as
the checker or as the timed CPU baseline.  The product path
(``decodekernels_b200``) never imports it and has no CPU fallback.

This is a numpy restatement of the reference's PyTorch oracles for the
``paged_attention_decode`` path (paths are inside the DecodeKernels project):

* ``gather_kv``            follows ``decode_kernels/reference.py:15-20``
* ``paged_attention_dense`` follows ``decode_kernels/reference.py:29-43``
* ``split_k_attention``    follows ``decode_kernels/reference.py:46-79``
  and also returns the per-partition statistics that the split-K kernel
  writes to its workspace (``csrc/paged_attention.cuh:214-220``): the
  normalised partial output ``o``, the max logit ``m`` and the exp-sum ``s``,
  stored at workspace row ``(seq * Hq + q_head) * P + p``.
* ``merge_partitions``     follows the log-sum-exp reduce
  ``csrc/paged_attention.cuh:229-269`` (``M = max m_i``,
  ``w_i = s_i * exp(m_i - M)``, ``out = sum w_i o_i / sum w_i``, zeros for
  empty sequences, ``num_parts = min(ceil(L / psize), P)``).

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors written by ``tests/golden/make_golden.py``, which runs
the reference's own ``reference.py`` / ``testing.py`` on seeded inputs.

All arithmetic is float32, like the reference (``q.float() * scale``,
``k.float()``, ``torch.softmax`` in fp32).  Inputs are numpy arrays; K/V
caches may be strided views ``[num_blocks, block_size, num_kv_heads, D]``.
"""

from __future__ import annotations

import math

import numpy as np


def _f32(x) -> np.ndarray:
    """float32 numpy view of a numpy array or a torch tensor (any 16-bit dtype)."""
    if hasattr(x, "detach"):  # torch tensor: numpy has no bfloat16
        x = x.detach().float().cpu().numpy()
    return np.asarray(x, dtype=np.float32)


def gather_kv(cache: np.ndarray, block_table_row: np.ndarray, seq_len: int) -> np.ndarray:
    """Rows ``[seq_len, num_kv_heads, D]`` of one sequence from a paged cache.

    Token ``t`` lives in physical block ``block_table_row[t // block_size]`` at
    offset ``t % block_size`` (reference.py:15-20; the kernel's ``kv_row_ptr``,
    paged_attention.cuh:62-71).
    """
    block_size = cache.shape[1]
    idx = np.arange(seq_len)
    blocks = np.asarray(block_table_row)[idx // block_size].astype(np.int64)
    return cache[blocks, idx % block_size]


def _per_seq_kv(k_cache, v_cache, block_tables, s, seq_len, group):
    """K and V of sequence ``s`` expanded to every query head: ``[L, Hq, D]``
    (reference.py:23-26, ``repeat_interleave(group, dim=1)``)."""
    k = np.repeat(gather_kv(k_cache, block_tables[s], seq_len), group, axis=1)
    v = np.repeat(gather_kv(v_cache, block_tables[s], seq_len), group, axis=1)
    return k, v


def _softmax_last(x: np.ndarray) -> np.ndarray:
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def paged_attention_dense(q, k_cache, v_cache, block_tables, seq_lens, scale=None) -> np.ndarray:
    """Dense softmax attention of each query token over its whole sequence.

    Returns float32 ``[num_seqs, Hq, D]``; empty sequences give zeros
    (reference.py:29-43).  The reference rounds its result to ``q.dtype``;
    callers that compare against it round with ``round_to``.
    """
    q, k_cache, v_cache = _f32(q), _f32(k_cache), _f32(v_cache)
    block_tables = np.asarray(block_tables)
    seq_lens = np.asarray(seq_lens)
    num_seqs, num_q_heads, head_dim = q.shape
    group = num_q_heads // k_cache.shape[2]
    scale = head_dim**-0.5 if scale is None else scale
    out = np.zeros((num_seqs, num_q_heads, head_dim), dtype=np.float32)
    for s in range(num_seqs):
        seq_len = int(seq_lens[s])
        if seq_len <= 0:
            continue
        k, v = _per_seq_kv(k_cache, v_cache, block_tables, s, seq_len, group)
        qs = q[s] * np.float32(scale)
        scores = np.einsum("hd,lhd->hl", qs, k)
        probs = _softmax_last(scores)
        out[s] = np.einsum("hl,lhd->hd", probs, v)
    return out


def split_k_attention(
    q, k_cache, v_cache, block_tables, seq_lens, scale=None, partition_size: int = 512, num_partitions: int | None = None
):
    """Flash-decoding math with per-partition statistics.

    Partition ``p`` of a sequence of length ``L`` covers tokens
    ``[p * partition_size, min((p + 1) * partition_size, L))``
    (paged_attention.cuh:89,109; reference.py:63-64).

    Returns ``(out, tmp_out, max_logits, exp_sums)``:

    * ``out``        float32 ``[n, Hq, D]``, the merged result (reference.py:73-78)
    * ``tmp_out``    float32 ``[n, Hq, P, D]``, normalised partial outputs
    * ``max_logits`` float32 ``[n, Hq, P]``, max scaled logit per partition
    * ``exp_sums``   float32 ``[n, Hq, P]``, ``sum exp(logit - max)`` per partition

    Partitions past a sequence's end hold NaN in the statistics arrays
    (the kernel never writes them and the merge never reads them).
    ``P`` defaults to ``ceil(max(seq_lens) / partition_size)``.
    """
    q, k_cache, v_cache = _f32(q), _f32(k_cache), _f32(v_cache)
    block_tables = np.asarray(block_tables)
    seq_lens = np.asarray(seq_lens)
    num_seqs, num_q_heads, head_dim = q.shape
    group = num_q_heads // k_cache.shape[2]
    scale = head_dim**-0.5 if scale is None else scale
    max_len = int(seq_lens[:num_seqs].max()) if num_seqs else 0
    P = num_partitions if num_partitions is not None else max(1, math.ceil(max_len / partition_size))
    out = np.zeros((num_seqs, num_q_heads, head_dim), dtype=np.float32)
    tmp_out = np.full((num_seqs, num_q_heads, P, head_dim), np.nan, dtype=np.float32)
    max_logits = np.full((num_seqs, num_q_heads, P), np.nan, dtype=np.float32)
    exp_sums = np.full((num_seqs, num_q_heads, P), np.nan, dtype=np.float32)
    for s in range(num_seqs):
        seq_len = int(seq_lens[s])
        if seq_len <= 0:
            continue
        k, v = _per_seq_kv(k_cache, v_cache, block_tables, s, seq_len, group)
        qs = q[s] * np.float32(scale)
        for p, start in enumerate(range(0, seq_len, partition_size)):
            if p >= P:
                break
            end = min(start + partition_size, seq_len)
            logits = np.einsum("hd,lhd->hl", qs, k[start:end])
            m = logits.max(axis=-1)
            e = np.exp(logits - m[:, None])
            ssum = e.sum(axis=-1)
            o = np.einsum("hl,lhd->hd", e, v[start:end]) / ssum[:, None]
            tmp_out[s, :, p] = o
            max_logits[s, :, p] = m
            exp_sums[s, :, p] = ssum
        out[s] = merge_partitions(
            tmp_out[s], max_logits[s], exp_sums[s], min(math.ceil(seq_len / partition_size), P)
        )
    return out, tmp_out, max_logits, exp_sums


def merge_partitions(tmp_out, max_logits, exp_sums, num_parts: int) -> np.ndarray:
    """Log-sum-exp merge of one sequence's partitions (paged_attention.cuh:241-268).

    ``tmp_out [Hq, P, D]``, ``max_logits`` / ``exp_sums`` ``[Hq, P]``; only the
    first ``num_parts`` partitions are read.  Returns float32 ``[Hq, D]``
    (zeros when ``num_parts <= 0``).
    """
    Hq, _, D = tmp_out.shape
    if num_parts <= 0:
        return np.zeros((Hq, D), dtype=np.float32)
    m = max_logits[:, :num_parts]
    s = exp_sums[:, :num_parts]
    gmax = m.max(axis=1, keepdims=True)
    w = s * np.exp(m - gmax)
    return (w[:, :, None] * tmp_out[:, :num_parts]).sum(axis=1) / w.sum(axis=1)[:, None]


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``float16`` / ``bfloat16`` (round to nearest even)
    and return them as float32, the way ``tensor.to(dtype)`` does."""
    x = np.asarray(x, dtype=np.float32)
    if dtype in ("float16", "fp16", "half"):
        return x.astype(np.float16).astype(np.float32)
    if dtype in ("bfloat16", "bf16"):
        bits = x.view(np.uint32).astype(np.uint64)
        rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
        nan = np.isnan(x)
        out = rounded.astype(np.uint32).view(np.float32).copy()
        out[nan] = np.nan
        return out
    if dtype in ("float32", "fp32"):
        return x
    raise ValueError(f"unknown dtype {dtype!r}")


def kv_bytes(seq_lens, num_kv_heads: int, head_dim: int, elem_size: int = 2) -> int:
    """K+V bytes one call must read: ``sum_s L_s * Hkv * D * 2 * esz``."""
    return int(sum(max(int(x), 0) for x in seq_lens)) * num_kv_heads * head_dim * 2 * elem_size
