"""Multi-GPU paged-attention decode on the GPUs of one node: KV-head
sharding (``ShardedPagedAttention``) and sequence sharding
(``SequenceShardedPagedAttention``).

KV-head sharding.

Attention is independent per KV head, and KV head ``h`` owns query heads
``[h*g, (h+1)*g)``.  Rank ``r`` of ``G`` therefore owns KV heads
``[r*Hkv/G, (r+1)*Hkv/G)``: their cache pages (its own
``[num_blocks, bs, Hkv/G, D]`` cache), the matching query heads and the
matching slice of the output.  Block tables and lengths are replicated.  No
data moves between ranks to compute a rank's heads, so a head-sharded
consumer (a tensor-parallel o_proj) needs no collective at all; an
all-gather of the per-head outputs is offered only for consumers that need
every head on every rank (``gather=True``): NCCL's, or ours over NVLink
peer memory (``exchange="p2p"``), where the decode's own output stores put
each rank's heads into every peer's receive buffer and one small kernel
completes the collective (``dk_paged_attention_decode_gather``;
``dk_gather_heads`` gathers outputs computed elsewhere).

Sequence sharding, for models whose KV heads cannot be split (MQA, or
fewer KV heads than GPUs) and for long contexts at small batch: block ``j``
of every sequence lives on rank ``j % G`` (block striping: balanced for any
length, and a sequence that grows never moves a page).  Every rank holds the
full query, computes fp32 partials ``(o, lse)`` over its own blocks
(``paged_attention_decode_lse``), and one NCCL all-gather of the packed
``[n, Hq, D + 4]`` rows lets every rank merge them with the log-sum-exp rule
(``merge_lse``) -- exact, since the token sets are disjoint.

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
    CPU oracle instead.  ``exchange`` chooses the gather: ``"nccl"``
    (``all_gather_into_tensor``) or ``"p2p"`` (over symmetric memory: fused
    into the decode with the native kernels, ``dk_paged_attention_decode_gather``,
    else ``dk_gather_heads`` after it; CUDA ranks of one node, waits bounded by
    ``wait_limit_ms``, 0 = 2 s).
    """

    _FLAG_BYTES = 256  # flag words at the head of each rank's symmetric buffer

    def __init__(self, num_q_heads: int, num_kv_heads: int, rank: int | None = None, world: int | None = None,
                 group=None, attention_fn: Callable | None = None, exchange: str = "nccl", wait_limit_ms: int = 0):
        import torch.distributed as dist

        if rank is None or world is None:
            if dist.is_available() and dist.is_initialized():
                rank, world = dist.get_rank(group), dist.get_world_size(group)
            else:
                rank, world = 0, 1
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', got {exchange!r}")
        self.shard = head_shard(num_q_heads, num_kv_heads, rank, world)
        self.group = group
        self.exchange = exchange
        self.wait_limit_ms = wait_limit_ms
        self._p2p = None
        self._native = attention_fn is None  # the sm_100a kernels: the gather can ride on the decode's stores
        if attention_fn is None:
            from .ops import paged_attention_decode

            attention_fn = paged_attention_decode
        self.attention_fn = attention_fn

    def _p2p_buffers(self, slot_bytes: int, device):
        """Symmetric allocation (collective on first use, or when a larger batch
        needs more room): every rank's [flags | 2 receive slots]."""
        if self._p2p is not None and self._p2p[0] >= slot_bytes:
            return self._p2p
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        group = self.group if self.group is not None else dist.group.WORLD
        buf = symm.empty(self._FLAG_BYTES + 2 * slot_bytes, dtype=torch.uint8, device=device)
        buf.zero_()
        hdl = symm.rendezvous(buf, group)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        base = [int(x) for x in hdl.buffer_ptrs]
        recv = [b + self._FLAG_BYTES for b in base]
        state = torch.zeros(4, dtype=torch.int32, device=device)
        self._p2p = (slot_bytes, buf, hdl, recv, base, state)
        return self._p2p

    def p2p_errors(self) -> int:
        """Peer waits that gave up (state word 3) since the buffers were made."""
        return 0 if self._p2p is None else int(self._p2p[5][3].item())

    def __call__(self, q_local, k_cache_local, v_cache_local, block_tables, seq_lens, scale=None, max_seq_len=None,
                 out=None, workspace=None, gather: bool = False, gathered_out=None) -> torch.Tensor:
        """This rank's heads ``[n, Hq/G, D]``, or with ``gather`` every head
        ``[n, Hq, D]`` (into ``gathered_out`` when given)."""
        s = self.shard
        if q_local.shape[1] != s.q_per_rank or k_cache_local.shape[2] != s.kv_per_rank:
            raise ValueError(
                f"rank {s.rank}: expected {s.q_per_rank} query heads and {s.kv_per_rank} KV heads locally, got "
                f"{q_local.shape[1]} and {k_cache_local.shape[2]}")
        if scale is None:
            scale = q_local.shape[-1] ** -0.5  # the full model's scale, not a per-shard one
        if gather and s.world > 1 and self.exchange == "p2p" and self._native:
            return self._decode_gather(q_local, k_cache_local, v_cache_local, block_tables, seq_lens, scale,
                                       max_seq_len, workspace, gathered_out)
        local = self.attention_fn(q_local, k_cache_local, v_cache_local, block_tables, seq_lens, scale=scale,
                                  max_seq_len=max_seq_len, out=out, workspace=workspace)
        if not gather or s.world == 1:
            return local
        return self.gather(local, gathered_out)

    def _decode_gather(self, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, workspace,
                       gathered_out):
        """Decode with the all-gather fused into the output stores
        (``dk_paged_attention_decode_gather``): every rank's rows go straight
        into every rank's receive slot; one small kernel then waits and copies."""
        from . import capi
        from .ops import alloc_workspace

        s = self.shard
        n, hpr, d = q.shape
        if max_seq_len is None:
            max_seq_len = int(seq_lens[:n].max().item()) if n > 0 else 0
        if gathered_out is None:
            gathered_out = torch.empty(n, s.num_q_heads, d, dtype=q.dtype, device=q.device)
        if workspace is None:
            workspace = alloc_workspace(n, hpr, d, max_seq_len, q.device, num_kv_heads=k_cache.shape[2],
                                        block_size=k_cache.shape[1], merge_counters=True)
        _, _, _, recv, flags, state = self._p2p_buffers(n * s.num_q_heads * d * q.element_size(), q.device)
        capi.decode_gather(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, workspace, recv, flags,
                           state, gathered_out, s.rank, s.world, self.wait_limit_ms)
        return gathered_out

    def gather(self, local: torch.Tensor, gathered_out: torch.Tensor | None = None) -> torch.Tensor:
        """Every rank's heads ``[n, Hq, D]`` from this rank's ``[n, Hq/G, D]``
        (a collective: every rank calls it with the same sizes)."""
        s = self.shard
        if s.world == 1:
            if gathered_out is None:
                return local
            gathered_out.copy_(local)
            return gathered_out
        if self.exchange == "p2p":
            from . import capi

            n, hpr, d = local.shape
            if gathered_out is None:
                gathered_out = torch.empty(n, s.num_q_heads, d, dtype=local.dtype, device=local.device)
            _, _, _, recv, flags, state = self._p2p_buffers(n * s.num_q_heads * d * local.element_size(),
                                                            local.device)
            capi.gather_heads(local, recv, flags, state, gathered_out, s.rank, s.world, self.wait_limit_ms)
            return gathered_out
        full = gather_heads(local, s, self.group)
        if gathered_out is not None:
            gathered_out.copy_(full)
            return gathered_out
        return full



def stripe_tables(block_tables: torch.Tensor, seq_lens: torch.Tensor, block_size: int, rank: int, world: int):
    """Rank ``rank``'s (block_tables, seq_lens) under block striping.

    Block ``j`` of a sequence belongs to rank ``j % world``; the rank's table
    row lists its blocks in order (contiguous int32 copy) and its length
    counts their tokens (the sequence's last block may be partial).  Works on
    CPU or device tensors; nothing leaves the device.  In a deployment each
    rank keeps only its own rows and pages; this helper derives them from a
    full table.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    bt = block_tables[:, rank::world].contiguous()
    L = seq_lens.to(torch.int64)
    nb = (L + block_size - 1) // block_size
    count = torch.clamp((nb - rank + world - 1) // world, min=0)
    owns_last = (nb > 0) & ((nb - 1) % world == rank)
    lens = count * block_size - torch.where(owns_last, nb * block_size - L, torch.zeros_like(L))
    return bt, lens.to(torch.int32)


def striped_max_len(max_seq_len: int, block_size: int, world: int) -> int:
    """Upper bound of any rank's striped length (host-side, graph-safe)."""
    blocks = -(-max_seq_len // block_size)
    return -(-blocks // world) * block_size


class SequenceShardedPagedAttention:
    """Decode attention over block-striped sequence shards, merged on every rank.

    ``lse_fn`` / ``merge_fn`` default to :func:`decodekernels_b200.paged_attention_decode_lse`
    and :func:`decodekernels_b200.merge_lse` (the sm_100a kernels); tests of
    the host-side logic on CPU ranks pass the CPU oracle instead.
    """

    def __init__(self, block_size: int, rank: int | None = None, world: int | None = None, group=None,
                 lse_fn: Callable | None = None, merge_fn: Callable | None = None, exchange: str = "nccl",
                 wait_limit_ms: int = 0):
        import torch.distributed as dist

        if rank is None or world is None:
            if dist.is_available() and dist.is_initialized():
                rank, world = dist.get_rank(group), dist.get_world_size(group)
            else:
                rank, world = 0, 1
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        self.rank, self.world, self.group, self.block_size = rank, world, group, block_size
        if lse_fn is None or merge_fn is None:
            from .ops import merge_lse, paged_attention_decode_lse

            lse_fn = lse_fn or paged_attention_decode_lse
            merge_fn = merge_fn or merge_lse
        self.lse_fn, self.merge_fn = lse_fn, merge_fn
        self._gather_buf = None
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', got {exchange!r}")
        self.exchange = exchange
        self.wait_limit_ms = wait_limit_ms
        self._p2p = None  # (block_floats, symmetric buffer, handle, recv ptrs, flag ptrs, state)

    def partial(self, q, k_cache_local, v_cache_local, block_tables_local, seq_lens_local, scale=None,
                max_seq_len=None, workspace=None, **cache_scales) -> torch.Tensor:
        """This rank's fp32 partial rows ``[n, Hq, D + 4]`` over its own blocks
        (``k_scale`` / ``v_scale`` keywords for e4m3 caches)."""
        if scale is None:
            scale = q.shape[-1] ** -0.5
        if max_seq_len is not None:
            max_seq_len = striped_max_len(max_seq_len, self.block_size, self.world)
        return self.lse_fn(q, k_cache_local, v_cache_local, block_tables_local, seq_lens_local, scale=scale,
                           max_seq_len=max_seq_len, workspace=workspace, **cache_scales)

    def gather(self, partial: torch.Tensor) -> torch.Tensor:
        """All-gather every rank's partial into ``[G, n, Hq, D + 4]`` (one
        collective; the result lands in this rank's own memory)."""
        import torch.distributed as dist

        if self.world == 1:
            return partial.unsqueeze(0)
        shape = (self.world, *partial.shape)
        if self._gather_buf is None or self._gather_buf.shape != shape or self._gather_buf.device != partial.device:
            self._gather_buf = torch.empty(shape, dtype=partial.dtype, device=partial.device)
        dist.all_gather_into_tensor(self._gather_buf.view(-1), partial.contiguous().view(-1), group=self.group)
        return self._gather_buf

    # ------------------------------------------------------------ peer memory
    _FLAG_FLOATS = 64  # flag words at the head of each rank's symmetric buffer (256 bytes)

    def _p2p_buffers(self, block_floats: int, device):
        """Symmetric allocation (collective on first use, or when a larger batch
        needs more room): every rank's [flags | 2 x world receive blocks]."""
        if self._p2p is not None and self._p2p[0] >= block_floats:
            return self._p2p
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        group = self.group if self.group is not None else dist.group.WORLD
        buf = symm.empty(self._FLAG_FLOATS + 2 * self.world * block_floats, dtype=torch.float32, device=device)
        buf.zero_()
        hdl = symm.rendezvous(buf, group)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        base = [int(x) for x in hdl.buffer_ptrs]
        flags = [b for b in base]
        recv = [b + 4 * self._FLAG_FLOATS for b in base]
        state = torch.zeros(4, dtype=torch.int32, device=device)
        self._p2p = (block_floats, buf, hdl, recv, flags, state)
        return self._p2p

    def p2p_errors(self) -> int:
        """Peer waits that gave up (state word 3) since the buffers were made."""
        return 0 if self._p2p is None else int(self._p2p[5][3].item())

    def __call__(self, q, k_cache_local, v_cache_local, block_tables_local, seq_lens_local, scale=None,
                 max_seq_len=None, out=None, workspace=None, k_scale: float = 1.0,
                 v_scale: float = 1.0) -> torch.Tensor:
        """Full attention output ``[n, Hq, D]`` (q's dtype) on every rank.

        ``max_seq_len`` is the longest WHOLE sequence (the local bound is
        derived from it); ``seq_lens_local`` / ``block_tables_local`` are this
        rank's striped lengths and blocks (:func:`stripe_tables`).
        """
        scales = {} if (k_scale, v_scale) == (1.0, 1.0) else {"k_scale": k_scale, "v_scale": v_scale}
        partial = self.partial(q, k_cache_local, v_cache_local, block_tables_local, seq_lens_local, scale,
                               max_seq_len, workspace, **scales)
        if self.exchange == "p2p" and self.world > 1:
            from . import capi

            n, hq, row = partial.shape
            _, _, _, recv, flags, state = self._p2p_buffers(n * hq * row, partial.device)
            if out is None:
                out = torch.empty(n, hq, row - 4, dtype=q.dtype, device=q.device)
            capi.exchange_merge_lse(partial, recv, flags, state, out, self.rank, self.world, self.wait_limit_ms)
            return out
        return self.merge_fn(self.gather(partial), out=out, dtype=q.dtype)
