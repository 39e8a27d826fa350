"""CPU oracle for sequence-sharded decode.  TEST INFRASTRUCTURE, NOT PRODUCT.

Only ``tests/`` and ``bench.py``'s parity check of the sequence-sharded
exchange may import this module, as the checker (and, in the CPU ``gloo``
tests of the sharding logic, as the stand-in for the CUDA kernels).

DecodeKernels runs on one GPU; splitting a sequence's tokens across GPUs is
new here, so this module restates the mathematics the split relies on, in
float32 numpy, on top of ``oracle.py``'s dense attention:

* ``attention_lse``: per (sequence, query head) the normalised output ``o``
  and ``lse = log(sum_t exp(scale * q . k_t))`` over the sequence's tokens
  (``o = 0``, ``lse = -inf`` when it has none) -- the same per-partition
  statistics the split-K workspace holds (``oracle.split_k_attention``), for
  a whole sequence.
* ``merge_lse``: for partials of disjoint token sets,
  ``M = max_r lse_r``, ``w_r = exp(lse_r - M)``,
  ``o = sum_r w_r o_r / sum_r w_r``, ``lse = M + log(sum_r w_r)`` -- the
  log-sum-exp merge of DecodeKernels' reduce kernel
  (``csrc/paged_attention.cuh:229-269``) with ``s_r exp(m_r)`` folded into
  ``exp(lse_r)``.
* ``stripe``: the block-striped split: block ``j`` of every sequence lives on
  rank ``j % world``, so rank ``r``'s table row is ``block_tables[s, r::world]``
  and its token count is that many blocks, the last one partial when the
  sequence's final block is ``r``'s.

Pinned by ``tests/test_sharded_lse_cpu.py``: merging the partials of any
stripe equals ``oracle.paged_attention_dense`` on the whole sequence.
"""

from __future__ import annotations

import numpy as np

from . import oracle


def attention_lse(q, k_cache, v_cache, block_tables, seq_lens, scale=None):
    """(o float32 [n, Hq, D], lse float32 [n, Hq])."""
    q, k_cache, v_cache = oracle._f32(q), oracle._f32(k_cache), oracle._f32(v_cache)
    block_tables = np.asarray(block_tables)
    seq_lens = np.asarray(seq_lens)
    n, hq, d = q.shape
    group = hq // k_cache.shape[2]
    scale = d**-0.5 if scale is None else scale
    o = np.zeros((n, hq, d), dtype=np.float32)
    lse = np.full((n, hq), -np.inf, dtype=np.float32)
    for s in range(n):
        L = int(seq_lens[s])
        if L <= 0:
            continue
        k, v = oracle._per_seq_kv(k_cache, v_cache, block_tables, s, L, group)
        scores = np.einsum("hd,lhd->hl", q[s] * np.float32(scale), k).astype(np.float64)
        m = scores.max(axis=-1, keepdims=True)
        e = np.exp(scores - m)
        tot = e.sum(axis=-1)
        o[s] = (np.einsum("hl,lhd->hd", e, v.astype(np.float64)) / tot[:, None]).astype(np.float32)
        lse[s] = (m[:, 0] + np.log(tot)).astype(np.float32)
    return o, lse


def merge_lse(o_parts, lse_parts):
    """Merge partials [R, n, Hq, D] / [R, n, Hq] of disjoint token sets."""
    o_parts = np.asarray(o_parts, dtype=np.float64)
    lse_parts = np.asarray(lse_parts, dtype=np.float64)
    m = lse_parts.max(axis=0)
    empty = ~np.isfinite(m)
    w = np.where(empty[None], 0.0, np.exp(lse_parts - np.where(empty, 0.0, m)[None]))
    tot = w.sum(axis=0)
    o = np.where(empty[..., None], 0.0, (w[..., None] * o_parts).sum(axis=0) / np.where(tot > 0, tot, 1.0)[..., None])
    lse = np.where(empty, -np.inf, m + np.log(np.where(tot > 0, tot, 1.0)))
    return o.astype(np.float32), lse.astype(np.float32)


def stripe(block_tables, seq_lens, block_size: int, rank: int, world: int):
    """Rank ``rank``'s (block_tables, seq_lens) under the block-striped split."""
    bt = np.asarray(block_tables)[:, rank::world]
    L = np.asarray(seq_lens, dtype=np.int64)
    nb = (L + block_size - 1) // block_size
    count = np.maximum(0, (nb - rank + world - 1) // world)
    owns_last = (nb > 0) & ((nb - 1) % world == rank)
    lens = count * block_size - np.where(owns_last, nb * block_size - L, 0)
    return np.ascontiguousarray(bt), lens.astype(np.int32)
