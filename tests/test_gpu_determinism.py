"""GPU: repeated calls on the same inputs give bit-identical outputs.

The decode has no atomics in its arithmetic (the merge order is fixed), so any
difference between two calls is a race.  The batches are made so that many
partitions end in a short last tile that some consumer warps have no rows of
-- the case in which a warp leaves its pipeline early -- on the e4m3 and the
16-bit TMA kernels, with the merge kernel and with the single-launch merge."""

import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import workloads

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

CALLS = 30


def _repeat(b, merge_counters):
    q, kv = b.q, b.kv
    n, hq, d = q.shape
    sc = b.config.kv_scale if b.config.kv_fp8 else 1.0
    ws = dk.alloc_workspace(n, hq, d, b.max_seq_len, "cuda", num_kv_heads=kv.k_cache.shape[2],
                            block_size=kv.block_size, merge_counters=merge_counters)
    outs = []
    for _ in range(CALLS):
        o = torch.empty_like(q)
        dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=b.max_seq_len,
                                  out=o, workspace=ws, k_scale=sc, v_scale=sc)
        outs.append(o)
    torch.cuda.synchronize()
    first = outs[0]
    assert not torch.isnan(first).any()
    for i, o in enumerate(outs[1:], 1):
        if not torch.equal(o, first):
            bad = (o != first).any(dim=-1).any(dim=-1).nonzero().flatten().tolist()
            raise AssertionError(f"call {i} differs from call 0 in sequences {bad[:8]} "
                                 f"(lengths {[b.lens[s] for s in bad[:8]]})")


@pytest.mark.parametrize("name", ["c4f8", "c4", "c2f8", "c2"])
@pytest.mark.parametrize("merge_counters", [False, True])
def test_repeated_calls_identical(name, merge_counters):
    b = workloads.make(name, "cuda")
    _repeat(b, merge_counters)
