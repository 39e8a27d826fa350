"""Seeded synthetic decode batches for the benchmark configs c1..c5.

Each config is a batch shape from the benchmark spec (the reference publishes
no dataset; every input is synthetic): sequence lengths drawn from
``torch.Generator().manual_seed(0)``, caches ~ N(0, sigma) in the config's
layout, block tables that are a seeded random permutation of the block pool
(no block shared).  Large caches are drawn on the target device.

``make(name, device, shard=(rank, world))`` builds rank ``rank``'s KV-head
shard for multi-GPU runs: that rank owns KV heads
``[rank * Hkv / world, (rank + 1) * Hkv / world)`` and the matching query
heads; lengths and block tables are the same on every rank.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .testing import PagedKV, make_paged_kv


@dataclass(frozen=True)
class Config:
    name: str
    description: str
    num_seqs: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    dtype: torch.dtype
    layout: str
    sigma: float = 1.0
    pool_blocks: int | None = None  # fixed block pool; None = exactly what the lengths need (+ spare)
    kv_fp8: bool = False  # caches hold e4m3 codes of the 16-bit draw, x / kv_scale
    kv_scale: float = 1.0

    @property
    def kv_bytes_per_elem(self) -> int:
        return 1 if self.kv_fp8 else torch.finfo(self.dtype).bits // 8


CONFIGS = {
    "c1": Config("c1", "CPU-runnable reference check: n=4, Hq32/Hkv8, D128, bs16, L={1,511,512,513}, bf16, NHD, "
                 "160-block pool", 4, 32, 8, 128, 16, torch.bfloat16, "nhd", pool_blocks=160),
    "c2": Config("c2", "Llama-3-8B-shaped decode batch: n=64, Hq32/Hkv8, D128, bs16, L~U[512,4096], fp16, vLLM "
                 "interleaved K|V, 20k-block pool", 64, 32, 8, 128, 16, torch.float16, "vllm", pool_blocks=20000),
    "c3": Config("c3", "Long-context split-K at batch 1: n=1, Hq64/Hkv8, D128, bs16, L=131072, bf16, HND, "
                 "8192-block pool", 1, 64, 8, 128, 16, torch.bfloat16, "hnd", pool_blocks=8192),
    "c4": Config("c4", "Head-dim-256 MQA: n=128, Hq8/Hkv1, D256, bs32, L~lognormal(median 2048, sigma 1) clipped "
                 "[1,32768], bf16 N(0,0.5), NHD", 128, 8, 1, 256, 32, torch.bfloat16, "nhd", sigma=0.5),
    "c5": Config("c5", "Mixed-length serving batch, KV-head sharded: n=256, Hq64/Hkv8, D128, bs16, L~U[1,32768] "
                 "with 5% empty, fp16, vLLM interleaved K|V", 256, 64, 8, 128, 16, torch.float16, "vllm"),
}


# FP8 (e4m3) variants: the same batches with per-tensor-scaled e4m3 caches
# (as reshape_and_cache writes them), half the KV bytes.
for _name in ("c2", "c3", "c4", "c5"):
    _c = CONFIGS[_name]
    CONFIGS[_name + "f8"] = Config(_name + "f8", _c.description + "; KV cache e4m3 (per-tensor scale 1/64)",
                                   _c.num_seqs, _c.num_q_heads, _c.num_kv_heads, _c.head_dim, _c.block_size, _c.dtype,
                                   _c.layout, _c.sigma, _c.pool_blocks, kv_fp8=True, kv_scale=1.0 / 64)


def seq_lens(name: str) -> list[int]:
    """The config's lengths, drawn from torch.Generator().manual_seed(0)."""
    name = name[:-2] if name.endswith("f8") else name
    g = torch.Generator().manual_seed(0)
    if name == "c1":
        return [1, 511, 512, 513]
    if name == "c2":
        return torch.randint(512, 4097, (64,), generator=g).tolist()
    if name == "c3":
        return [131072]
    if name == "c4":
        x = torch.empty(128, dtype=torch.float64).log_normal_(mean=math.log(2048.0), std=1.0, generator=g)
        return x.round().clamp(1, 32768).to(torch.int64).tolist()
    if name == "c5":
        lens = torch.randint(1, 32769, (256,), generator=g)
        empty = torch.randperm(256, generator=g)[: round(0.05 * 256)]
        lens[empty] = 0
        return lens.tolist()
    raise KeyError(name)


@dataclass
class Batch:
    config: Config
    q: torch.Tensor
    kv: PagedKV
    lens: list[int]
    rank: int = 0
    world: int = 1
    kv_heads: int = field(default=0)

    @property
    def max_seq_len(self) -> int:
        return max(self.lens) if self.lens else 0

    def kv_bytes(self) -> int:
        """K+V bytes this batch's call must read: sum L * Hkv_local * D * 2 * esz."""
        esz = self.config.kv_bytes_per_elem
        return sum(self.lens) * self.kv_heads * self.config.head_dim * 2 * esz

    def algorithmic_bytes(self) -> int:
        """K+V once + q in + out + block-table entries + seq_lens (int32)."""
        c = self.config
        esz = torch.finfo(c.dtype).bits // 8  # q and out
        hq = self.q.shape[1]
        tables = sum(-(-L // c.block_size) for L in self.lens) * 4
        return self.kv_bytes() + 2 * len(self.lens) * hq * c.head_dim * esz + tables + 4 * len(self.lens)


def _to_e4m3(buf: torch.Tensor, scale: float) -> torch.Tensor:
    """uint8 e4m3 codes of sat(buf / scale), converted in slices of the first
    dimension to bound the temporary float32 memory."""
    out = torch.empty(buf.shape, dtype=torch.uint8, device=buf.device)
    step = max(1, buf.shape[0] * (64 << 20) // max(buf.numel(), 1))
    for i in range(0, buf.shape[0], step):
        x = buf[i : i + step].float().div_(scale).clamp_(-448.0, 448.0)
        out[i : i + step] = x.to(torch.float8_e4m3fn).view(torch.uint8)
    return out


def _layout_views(buf: torch.Tensor, layout: str, head_dim: int):
    """K, V views [blocks, bs, heads, D] of a freshly drawn buffer."""
    if layout == "nhd":
        return buf[0], buf[1]
    if layout == "hnd":
        return buf[0].transpose(1, 2), buf[1].transpose(1, 2)
    if layout == "vllm":
        k, v = buf.transpose(1, 2).split(head_dim, dim=-1)
        return k, v
    raise ValueError(layout)


def make_striped(name: str, device="cuda", stripe: tuple[int, int] = (0, 1), seed: int = 0) -> Batch:
    """Rank ``rank``'s part of config ``name`` under sequence (block-striped)
    sharding over ``world`` GPUs: block ``j`` of every sequence lives on rank
    ``j % world``.  The rank holds the whole query batch (all heads, the same
    draw on every rank), only its own blocks (a compact pool with its own
    block tables) and its striped lengths.  ``Batch.lens`` are those local
    lengths, so ``kv_bytes`` is what this rank reads."""
    c = CONFIGS[name]
    rank, world = stripe
    bs, d, hkv = c.block_size, c.head_dim, c.num_kv_heads
    full = seq_lens(name)
    nblk = [-(-L // bs) for L in full]
    mine = [len(range(rank, nb, world)) for nb in nblk]
    lens = []
    for L, nb, cnt in zip(full, nblk, mine):
        last_mine = nb > 0 and (nb - 1) % world == rank
        lens.append(cnt * bs - (nb * bs - L if last_mine else 0))
    need = sum(mine)
    pool = need + 16
    gen = torch.Generator(device=device).manual_seed(seed * 1000 + 100 + rank)
    if c.layout == "vllm":
        buf = torch.randn(pool, hkv, bs, 2 * d, generator=gen, device=device, dtype=c.dtype)
    elif c.layout == "hnd":
        buf = torch.randn(2, pool, hkv, bs, d, generator=gen, device=device, dtype=c.dtype)
    else:
        buf = torch.randn(2, pool, bs, hkv, d, generator=gen, device=device, dtype=c.dtype)
    if c.sigma != 1.0:
        buf.mul_(c.sigma)
    if c.kv_fp8:
        buf = _to_e4m3(buf, c.kv_scale)
    k, v = _layout_views(buf, c.layout, d)
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(seed + 7 + rank)).to(torch.int32)
    width = max(max(mine) if mine else 1, 1)
    tables = torch.zeros(len(full), width, dtype=torch.int32)
    off = 0
    for i, cnt in enumerate(mine):
        tables[i, :cnt] = perm[off : off + cnt]
        off += cnt
    qg = torch.Generator(device=device).manual_seed(seed * 1000 + 500)  # same query on every rank
    q = torch.randn(len(full), c.num_q_heads, d, generator=qg, device=device, dtype=c.dtype)
    kv = PagedKV(k, v, tables.to(device), torch.tensor(lens, dtype=torch.int32, device=device), bs)
    return Batch(c, q, kv, lens, rank, world, hkv)


def make(name: str, device="cuda", shard: tuple[int, int] = (0, 1), seed: int = 0,
         seqs: list[int] | None = None) -> Batch:
    """Build config ``name`` (or only sequences ``seqs`` of it) on ``device``;
    ``shard = (rank, world)`` keeps rank ``rank``'s KV heads (head sharding)."""
    c = CONFIGS[name]
    rank, world = shard
    if c.num_kv_heads % world:
        raise ValueError(f"{name}: {c.num_kv_heads} KV heads cannot be split over {world} GPUs")
    hkv = c.num_kv_heads // world
    hq = c.num_q_heads // world
    lens = seq_lens(name)
    if seqs is not None:
        lens = [lens[i] for i in seqs]
    if name == "c1" and world == 1 and seqs is None:
        # the reference fixture builder's exact draw (CPU generator), as in the golden vectors
        kv = make_paged_kv(lens, hkv, c.head_dim, c.block_size, c.dtype, device, layout=c.layout,
                           extra_blocks=c.pool_blocks - sum(-(-L // c.block_size) for L in lens), seed=seed)
        g = torch.Generator().manual_seed(1)
        q = torch.randn(len(lens), hq, c.head_dim, generator=g, dtype=c.dtype).to(device)
        return Batch(c, q, kv, lens, rank, world, hkv)

    bs, d = c.block_size, c.head_dim
    nblk = [-(-L // bs) for L in lens]
    need = sum(nblk)
    pool = max(c.pool_blocks or 0, need + 16) if seqs is None else need + 16
    gen = torch.Generator(device=device).manual_seed(seed * 1000 + rank)
    if c.layout == "vllm":
        buf = torch.randn(pool, hkv, bs, 2 * d, generator=gen, device=device, dtype=c.dtype)
    elif c.layout == "hnd":
        buf = torch.randn(2, pool, hkv, bs, d, generator=gen, device=device, dtype=c.dtype)
    else:
        buf = torch.randn(2, pool, bs, hkv, d, generator=gen, device=device, dtype=c.dtype)
    if c.sigma != 1.0:
        buf.mul_(c.sigma)
    if c.kv_fp8:
        buf = _to_e4m3(buf, c.kv_scale)
    k, v = _layout_views(buf, c.layout, d)
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(seed + 7)).to(torch.int32)
    width = max(max(nblk) if nblk else 1, 1)
    tables = torch.zeros(len(lens), width, dtype=torch.int32)
    off = 0
    for i, nb in enumerate(nblk):
        tables[i, :nb] = perm[off : off + nb]
        off += nb
    qg = torch.Generator(device=device).manual_seed(seed * 1000 + 500 + rank)
    q = torch.randn(len(lens), hq, d, generator=qg, device=device, dtype=c.dtype)
    kv = PagedKV(k, v, tables.to(device), torch.tensor(lens, dtype=torch.int32, device=device), bs)
    return Batch(c, q, kv, lens, rank, world, hkv)


def compact_sequences(batch: Batch, seqs: list[int]):
    """Copy sequences ``seqs`` of a device batch to the host as a compact NHD
    cache (their pages only) with fresh block tables -- used to check a few
    sequences of a huge batch against the CPU oracle."""
    kv, bs = batch.kv, batch.config.block_size
    ks, vs, rows = [], [], []
    base = 0
    width = 1
    for s in seqs:
        nb = -(-batch.lens[s] // bs)
        ids = kv.block_tables[s, :nb].long()
        ks.append(kv.k_cache[ids].cpu())
        vs.append(kv.v_cache[ids].cpu())
        rows.append(list(range(base, base + nb)))
        base += nb
        width = max(width, nb)
    k = torch.cat(ks) if ks else torch.zeros(0)
    v = torch.cat(vs) if vs else torch.zeros(0)
    tables = torch.zeros(len(seqs), width, dtype=torch.int32)
    for i, r in enumerate(rows):
        if r:
            tables[i, : len(r)] = torch.tensor(r, dtype=torch.int32)
    lens = torch.tensor([batch.lens[s] for s in seqs], dtype=torch.int32)
    return batch.q[seqs].cpu(), PagedKV(k, v, tables, lens, bs)


def dequantize(kv: PagedKV, config: Config) -> PagedKV:
    """For an e4m3 config, the same cache as ``config.dtype`` values
    (code * kv_scale; exact for the power-of-two scale used here), e.g. to
    check a batch against a 16-bit reference; other configs unchanged."""
    if not config.kv_fp8:
        return kv

    def deq(c):
        return (c.view(torch.float8_e4m3fn).to(torch.float32) * config.kv_scale).to(config.dtype)

    return PagedKV(deq(kv.k_cache), deq(kv.v_cache), kv.block_tables, kv.seq_lens, kv.block_size)
