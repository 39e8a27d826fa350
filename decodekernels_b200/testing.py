"""Paged KV-cache builders for tests and benchmarks.

``make_paged_kv`` keeps the signature and the seeded semantics of the
reference's fixture builder (DecodeKernels ``decode_kernels/testing.py:23-77``):
for the same arguments it returns bit-identical caches, block tables and
lengths, which is what lets the golden vectors produced by the reference's own
oracle be replayed here without the reference installed.  The golden tests
check that by hashing the generated tensors.

Layouts (all returned as ``[num_blocks, block_size, num_kv_heads, head_dim]``
views with ``head_dim`` contiguous):

* ``nhd``  contiguous NHD (FlashInfer NHD)
* ``hnd``  stored ``[num_blocks, num_kv_heads, block_size, head_dim]`` and
  viewed as NHD (FlashInfer HND)
* ``vllm`` one interleaved buffer ``[num_blocks, num_kv_heads, block_size,
  2 * head_dim]`` viewed as two strided NHD tensors, K first, V ``head_dim``
  elements later
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class PagedKV:
    k_cache: torch.Tensor  # [num_blocks, block_size, num_kv_heads, head_dim], possibly a strided view
    v_cache: torch.Tensor
    block_tables: torch.Tensor  # [num_seqs, max_blocks] int32
    seq_lens: torch.Tensor  # [num_seqs] int32
    block_size: int

    @property
    def max_seq_len(self) -> int:
        return int(self.seq_lens.max().item()) if self.seq_lens.numel() else 0


def _random_layout(shape_nhd, layout: str, gen: torch.Generator, dtype, device):
    """Two K/V views in ``layout``, drawn from ``gen`` in the reference's order."""
    nb, bs, h, d = shape_nhd
    if layout == "nhd":
        k = torch.randn(nb, bs, h, d, generator=gen, dtype=dtype)
        v = torch.randn(nb, bs, h, d, generator=gen, dtype=dtype)
        return k.to(device), v.to(device)
    if layout == "hnd":
        k = torch.randn(nb, h, bs, d, generator=gen, dtype=dtype)
        v = torch.randn(nb, h, bs, d, generator=gen, dtype=dtype)
        return k.to(device).transpose(1, 2), v.to(device).transpose(1, 2)
    if layout == "vllm":
        kv = torch.randn(nb, h, bs, 2 * d, generator=gen, dtype=dtype).to(device)
        k, v = kv.transpose(1, 2).split(d, dim=-1)
        return k, v
    raise ValueError(f"unknown layout {layout!r}")


def make_paged_kv(
    seq_lens: list[int],
    num_kv_heads: int,
    head_dim: int,
    block_size: int = 16,
    dtype: torch.dtype = torch.float16,
    device: str | torch.device = "cpu",
    layout: str = "nhd",
    extra_blocks: int = 3,
    seed: int = 0,
) -> PagedKV:
    """Random paged KV cache whose physical blocks are a seeded permutation.

    Sequence ``s`` owns ``ceil(L_s / block_size)`` blocks, taken in order
    from one random permutation of all ``sum + extra_blocks`` blocks, so no
    block is shared and every table row points at scattered blocks.  Unused
    table entries are 0.
    """
    gen = torch.Generator(device="cpu").manual_seed(seed)
    nblk = [-(-int(n) // block_size) for n in seq_lens]
    num_blocks = sum(nblk) + extra_blocks
    k, v = _random_layout((num_blocks, block_size, num_kv_heads, head_dim), layout, gen, dtype, device)
    perm = torch.randperm(num_blocks, generator=gen)
    width = max(max(nblk) if nblk else 1, 1)
    tables = torch.zeros(len(seq_lens), width, dtype=torch.int32)
    offset = 0
    for row, count in enumerate(nblk):
        tables[row, :count] = perm[offset : offset + count].to(torch.int32)
        offset += count
    return PagedKV(
        k_cache=k,
        v_cache=v,
        block_tables=tables.to(device),
        seq_lens=torch.tensor(list(seq_lens), dtype=torch.int32, device=device),
        block_size=block_size,
    )


def make_queries(num_seqs: int, num_q_heads: int, head_dim: int, dtype=torch.float16, seed: int = 1, device="cpu"):
    """Seeded query batch ``[num_seqs, num_q_heads, head_dim]`` drawn on the CPU
    (the reference tests' ``_queries`` helper, tests/test_reference.py:25-27)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(num_seqs, num_q_heads, head_dim, generator=g, dtype=dtype).to(device)


def tensor_digest(t: torch.Tensor) -> str:
    """sha256 of a tensor's logical contents (row-major, raw bytes).

    Used to prove that two processes built the same inputs."""
    import hashlib

    c = t.detach().contiguous().cpu()
    if c.dtype in (torch.float16, torch.bfloat16):
        c = c.view(torch.int16)
    return hashlib.sha256(c.numpy().tobytes()).hexdigest()
