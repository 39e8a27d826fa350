"""Replays the golden cases written by ``tests/golden/make_golden.py``.

``load_cases()`` returns the case metadata; ``build(case, device)`` rebuilds
the exact inputs with ``decodekernels_b200.testing`` and checks their sha256
digests against the ones recorded from the reference's own fixture builder,
so every comparison below is on the same inputs the reference saw.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from decodekernels_b200.testing import make_paged_kv, tensor_digest

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def load_cases() -> list[dict]:
    return json.loads((GOLDEN / "cases.json").read_text())["cases"]


def case_by_name(name: str) -> dict:
    for c in load_cases():
        if c["name"] == name:
            return c
    raise KeyError(name)


def outputs(case: dict) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{case['name']}.npz") as z:
        return {k: z[k] for k in z.files}


def build(case: dict, device="cpu", check_digests: bool = True):
    """Rebuild ``(q, PagedKV)`` for a case on ``device``."""
    dtype = DTYPES[case["dtype"]]
    kv = make_paged_kv(case["seq_lens"], case["num_kv_heads"], case["head_dim"], case["block_size"], dtype, "cpu",
                       layout=case["layout"], extra_blocks=case["extra_blocks"], seed=case["seed"])
    g = torch.Generator().manual_seed(case["q_seed"])
    q = torch.randn(len(case["seq_lens"]), case["num_q_heads"], case["head_dim"], generator=g, dtype=dtype)
    if check_digests:
        got = {
            "k_cache": tensor_digest(kv.k_cache),
            "v_cache": tensor_digest(kv.v_cache),
            "block_tables": tensor_digest(kv.block_tables),
            "seq_lens": tensor_digest(kv.seq_lens),
            "q": tensor_digest(q),
        }
        assert got == case["digests"], f"{case['name']}: rebuilt inputs differ from the golden inputs"
        assert list(kv.k_cache.stride()) == case["k_strides"]
    if str(device) != "cpu":
        kv = _to_device(kv, case, device)
        q = q.to(device)
    return q, kv


def _to_device(kv, case, device):
    """Move a CPU PagedKV to ``device`` keeping its layout (views stay views)."""
    layout = case["layout"]
    if layout == "nhd":
        k, v = kv.k_cache.to(device), kv.v_cache.to(device)
    elif layout == "hnd":
        k = kv.k_cache.transpose(1, 2).contiguous().to(device).transpose(1, 2)
        v = kv.v_cache.transpose(1, 2).contiguous().to(device).transpose(1, 2)
    else:  # vllm: K and V are views of one interleaved buffer
        d = case["head_dim"]
        base = torch.cat([kv.k_cache, kv.v_cache], dim=-1).transpose(1, 2).contiguous().to(device)
        k, v = base.transpose(1, 2).split(d, dim=-1)
    kv.k_cache, kv.v_cache = k, v
    kv.block_tables = kv.block_tables.to(device)
    kv.seq_lens = kv.seq_lens.to(device)
    return kv
