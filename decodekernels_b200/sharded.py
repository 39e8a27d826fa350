"""KV-head sharding of paged-attention decode across the GPUs of one node.

Attention is independent per KV head, and KV head ``h`` owns query heads
``[h*g, (h+1)*g)``.  Rank ``r`` of ``G`` therefore owns KV heads
``[r*Hkv/G, (r+1)*Hkv/G)``: their cache pages (its own
``[num_blocks, bs, Hkv/G, D]`` cache), the matching query heads and the
matching slice of the output.  Block tables and lengths are replicated.  No
data moves between ranks to compute a rank's heads, so a head-sharded
consumer (a tensor-parallel o_proj) needs no collective at all; an NCCL
all-gather of the per-head outputs is offered only for consumers that need
every head on every rank (``gather=True``).

The reference has no multi-GPU code; this layer is new.  Ranks are one
process per GPU (``torch.distributed``, NCCL over NVLink/NVSwitch); the
host-side logic is covered with CPU ``gloo`` ranks in the tests.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch


@dataclass(frozen=True)
class HeadShard:
    """The heads rank ``rank`` of ``world`` owns."""

    rank: int
    world: int
    num_q_heads: int
    num_kv_heads: int

    @property
    def kv_per_rank(self) -> int:
        return self.num_kv_heads // self.world

    @property
    def q_per_rank(self) -> int:
        return self.num_q_heads // self.world

    @property
    def kv_slice(self) -> slice:
        return slice(self.rank * self.kv_per_rank, (self.rank + 1) * self.kv_per_rank)

    @property
    def q_slice(self) -> slice:
        return slice(self.rank * self.q_per_rank, (self.rank + 1) * self.q_per_rank)


def head_shard(num_q_heads: int, num_kv_heads: int, rank: int, world: int) -> HeadShard:
    """Validate and describe rank ``rank``'s shard.

    Raises ValueError when the KV heads cannot be split evenly (for example
    MQA with one KV head on more than one GPU: run replicas instead)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_kv_heads <= 0 or num_q_heads % num_kv_heads:
        raise ValueError("num_q_heads must be a positive multiple of num_kv_heads")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads cannot be split over {world} ranks")
    return HeadShard(rank, world, num_q_heads, num_kv_heads)


def shard_queries(q: torch.Tensor, shard: HeadShard) -> torch.Tensor:
    """This rank's query heads of a full ``[n, Hq, D]`` batch (a view)."""
    return q[:, shard.q_slice]


def shard_cache(cache: torch.Tensor, shard: HeadShard) -> torch.Tensor:
    """This rank's heads of a full ``[num_blocks, bs, Hkv, D]`` cache view (a
    strided view, read in place).  In a real deployment each rank allocates
    only its own heads' pages; this helper exists for tests and tools that
    hold the whole cache."""
    return cache[:, :, shard.kv_slice]


def gather_heads(local_out: torch.Tensor, shard: HeadShard, group=None) -> torch.Tensor:
    """All-gather the per-rank outputs ``[n, Hq/G, D]`` into ``[n, Hq, D]`` on
    every rank (one ``all_gather_into_tensor``; the result lands in this
    rank's own memory)."""
    import torch.distributed as dist

    n, hq_l, d = local_out.shape
    buf = torch.empty(shard.world * n * hq_l * d, dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(buf, local_out.contiguous().view(-1), group=group)
    return buf.view(shard.world, n, hq_l, d).permute(1, 0, 2, 3).reshape(n, shard.world * hq_l, d)


class ShardedPagedAttention:
    """Decode attention for this rank's KV heads, optionally gathered.

    ``attention_fn`` defaults to :func:`decodekernels_b200.paged_attention_decode`
    (the sm_100a kernels); tests of the host-side logic on CPU ranks pass the
    CPU oracle instead.
    """

    def __init__(self, num_q_heads: int, num_kv_heads: int, rank: int | None = None, world: int | None = None,
                 group=None, attention_fn: Callable | None = None):
        import torch.distributed as dist

        if rank is None or world is None:
            if dist.is_available() and dist.is_initialized():
                rank, world = dist.get_rank(group), dist.get_world_size(group)
            else:
                rank, world = 0, 1
        self.shard = head_shard(num_q_heads, num_kv_heads, rank, world)
        self.group = group
        if attention_fn is None:
            from .ops import paged_attention_decode

            attention_fn = paged_attention_decode
        self.attention_fn = attention_fn

    def __call__(self, q_local, k_cache_local, v_cache_local, block_tables, seq_lens, scale=None, max_seq_len=None,
                 out=None, workspace=None, gather: bool = False) -> torch.Tensor:
        s = self.shard
        if q_local.shape[1] != s.q_per_rank or k_cache_local.shape[2] != s.kv_per_rank:
            raise ValueError(
                f"rank {s.rank}: expected {s.q_per_rank} query heads and {s.kv_per_rank} KV heads locally, got "
                f"{q_local.shape[1]} and {k_cache_local.shape[2]}")
        if scale is None:
            scale = q_local.shape[-1] ** -0.5  # the full model's scale, not a per-shard one
        local = self.attention_fn(q_local, k_cache_local, v_cache_local, block_tables, seq_lens, scale=scale,
                                  max_seq_len=max_seq_len, out=out, workspace=workspace)
        if not gather or s.world == 1:
            return local
        return gather_heads(local, s, self.group)
