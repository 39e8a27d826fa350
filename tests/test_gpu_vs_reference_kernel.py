"""GPU: this library against the reference's own kernels on the benchmark
configs, on identical device inputs.

The reference kernels are compiled from the DecodeKernels source tree by
oracle/build.py (oracle/_ref/libdk_ref_kernel.so).  Both run on the same
caches; outputs must agree within the spec's tolerance, and both are timed
with CUDA events (L2 flushed before each call).  Timings are printed and, when
DK_PERF_LOG names a file, appended to it as JSON lines; they are reported,
not asserted.
"""

import json
import os

import numpy as np
import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import workloads
from oracle import native

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
    pytest.mark.skipif(not native.have_reference_kernel(), reason="reference kernel not built (oracle/_ref)"),
]


def _time(fn, iters=20, warmup=3):
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    st = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    en = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for i in range(iters):
        flush.zero_()
        st[i].record()
        fn()
        en[i].record()
    torch.cuda.synchronize()
    us = sorted(s.elapsed_time(e) * 1e3 for s, e in zip(st, en))
    return us[len(us) // 2]


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_matches_and_times_reference_kernel(name):
    b = workloads.make(name, "cuda")
    q, kv = b.q, b.kv
    n, hq, d = q.shape
    L = b.max_seq_len
    scale = d**-0.5
    ours = torch.empty_like(q)
    ws = dk.alloc_workspace(n, hq, d, L, "cuda", num_kv_heads=kv.k_cache.shape[2], block_size=kv.block_size)
    ref = torch.empty_like(q)
    ref_ws = native.reference_workspace(n, hq, d, L, "cuda")

    def run_ours():
        dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=L, out=ours,
                                  workspace=ws)

    def run_ref():
        native.reference_kernel(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale, L, ref, ref_ws)

    run_ours()
    run_ref()
    torch.cuda.synchronize()
    diff = (ours.float() - ref.float()).abs()
    assert torch.isfinite(ours).all()
    assert diff.max().item() <= 2e-2 and diff.mean().item() <= 2e-3, (diff.max().item(), diff.mean().item())

    t_ours = _time(run_ours)
    t_ref = _time(run_ref)
    kvb = b.kv_bytes()
    rec = {"workload": name, "kv_bytes": kvb, "ours_us": t_ours, "ref_us": t_ref, "speedup": t_ref / t_ours,
           "ours_TBps": kvb / t_ours / 1e6, "ref_TBps": kvb / t_ref / 1e6, "max_abs_diff": diff.max().item()}
    print(json.dumps(rec))
    path = os.environ.get("DK_PERF_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(rec) + "\n")
    del b, kv
    torch.cuda.empty_cache()
