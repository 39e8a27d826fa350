"""GPU: the partition size fitted on the device to each batch's lengths.

For e4m3 caches and batches of a few (sequence, KV head) pairs -- at most one
per SM -- the planner's size only bounds the partition kernel's choice:
every CTA of the compact grid picks the smallest multiple of the kernel's
tile, down to DkPlan.fit_min_partition, whose live items fit one wave of
resident CTAs (the planned size when even its items do not fit), and the
merge kernel reads it from a workspace row no partition reaches.  Each case
predicts that size on the host from the lengths and the plan's occupancy,
and requires the fitted call to be bit-identical to a call with the
predicted size fixed (any other size gives other partial sums), and close to
the oracle.  A captured CUDA graph must refit on every replay, from the
lengths in device memory at that time.  16-bit caches keep the planned size.
"""

import numpy as np
import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import capi
from decodekernels_b200.testing import make_paged_kv
from gpu_helpers import alloc_ws, assert_attention_close, fp8_caches, oracle_dense, oracle_dense_fp8

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

KS, VS = 0.02, 0.015
MAX_LEN = 32768


def _lognormal_lens(n, seed, median=2048, sigma=1.0, zeros=()):
    """c4's spread: lognormal lengths clipped to [1, MAX_LEN] (and some empty)."""
    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(rng.lognormal(np.log(median), sigma, n)), 1, MAX_LEN).astype(int)
    lens[list(zeros)] = 0
    return lens.tolist()


def _gran(fp8, d):
    """Tokens per tile of the e4m3 partition kernel, the unit of a fitted
    size: 4 consumer warps x two 16-token slices at head_dim 128, 2 warps x
    one slice at 256."""
    return 128 if d == 128 else 32


def _predicted(lens, hkv, plan, gran):
    slots = plan["ctas_per_sm"] * torch.cuda.get_device_properties(0).multi_processor_count

    def items(ps):
        return hkv * sum(max(1, -(-min(max(l, 0), MAX_LEN) // ps)) for l in lens)

    hi, lo = plan["partition_size"], plan["fit_min_partition"]
    if items(hi) > slots:
        return hi
    return min(ps for ps in range(lo, hi + 1, gran) if items(ps) <= slots)


def _call(q, kv, k, v, ps, counters, fp8):
    n, hq, d = q.shape
    hkv = k.shape[2]
    parts = -(-MAX_LEN // ps) if ps else capi.num_partitions(n, hkv, d, kv.block_size, MAX_LEN)
    ws = alloc_ws(n, hq, d, parts, q.device)
    flags = 0
    if counters:
        ws = (*ws, torch.zeros(n * hkv, dtype=torch.int32, device=q.device))
        flags = capi.DK_FLAG_FORCE_FUSED_MERGE
    scales = (KS, VS) if fp8 else (1.0, 1.0)
    out = torch.full_like(q, float("nan"))
    plan = capi.plan(q, k, v, kv.block_tables, kv.seq_lens, d**-0.5, MAX_LEN, out, ws, ps, False, flags, *scales)
    capi.decode(q, k, v, kv.block_tables, kv.seq_lens, d**-0.5, MAX_LEN, out, ws, ps, False, flags=flags,
                k_scale=scales[0], v_scale=scales[1])
    torch.cuda.synchronize()
    return out, plan


@pytest.mark.parametrize(
    "dtype,d,hkv,group,layout,bs,n,merge",
    [
        (torch.bfloat16, 256, 1, 8, "nhd", 32, 96, "kernel"),  # c4's shape at 96 sequences
        (torch.bfloat16, 256, 1, 8, "hnd", 32, 96, "fused"),   # ... one launch (merge counters)
        (torch.float16, 128, 2, 8, "vllm", 16, 64, "kernel"),  # 128-token tiles, interleaved K|V
        (torch.float16, 128, 2, 4, "vllm", 16, 64, "fused"),
    ],
)
def test_fitted_size_is_the_predicted_one(dtype, d, hkv, group, layout, bs, n, merge):
    lens = _lognormal_lens(n, seed=d + n + hkv, zeros=(3, 40))
    kv = make_paged_kv(lens, hkv, d, bs, dtype, "cuda", layout=layout, seed=n)
    g = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn(n, hkv * group, d, generator=g, device="cuda", dtype=torch.float32).to(dtype)
    k, v = fp8_caches(kv, layout, KS, VS)
    fitted, plan = _call(q, kv, k, v, 0, merge == "fused", True)
    assert plan["path"] == capi.DK_PATH_TMA_MMA and plan["fit_min_partition"] == 512, plan
    assert plan["num_partitions"] == MAX_LEN // 512 + 1 and plan["ctas_per_sm"] > 0  # + the size's row
    ps = _predicted(lens, hkv, plan, _gran(True, d))
    assert 512 <= ps < plan["partition_size"], (ps, plan)  # these lengths fit below the planned size
    fixed, fplan = _call(q, kv, k, v, ps, merge == "fused", True)
    assert fplan["fit_min_partition"] == 0 and fplan["partition_size"] == ps
    assert torch.equal(fitted, fixed), f"fitted call differs from partition_size={ps}"
    assert_attention_close(fitted, oracle_dense_fp8(q, kv, k, v, KS, VS), dtype, f"fitted ({ps} tokens)")
    assert capi.wait_timeouts(0) == 0


def test_sixteen_bit_caches_keep_the_planned_size():
    n, hkv, group, d = 96, 1, 8, 256
    lens = _lognormal_lens(n, seed=4)
    kv = make_paged_kv(lens, hkv, d, 32, torch.bfloat16, "cuda", seed=4)
    q = torch.randn(n, hkv * group, d, device="cuda", dtype=torch.bfloat16)
    out, plan = _call(q, kv, kv.k_cache, kv.v_cache, 0, False, False)
    assert plan["fit_min_partition"] == 0 and plan["num_partitions"] == -(-MAX_LEN // plan["partition_size"])
    assert_attention_close(out, oracle_dense(q, kv), torch.bfloat16, "16-bit, planned size")


@pytest.mark.parametrize("n,step", [(24, 37), (37, 0)])
def test_lengths_near_the_bound_keep_the_planned_size(n, step):
    # every sequence near max_seq_len: the planned size's items exceed a wave,
    # so the device keeps it (and the CTAs of one wave loop over the items).
    # 37 sequences of 32768 tokens: some size above the planned one would fit
    # the wave (43 tiles of 128 tokens, 222 items per KV head at 3 CTAs per
    # SM), and the device must not pick it.
    hkv, group, d = 2, 8, 128
    lens = [MAX_LEN - step * i for i in range(n)]
    kv = make_paged_kv(lens, hkv, d, 16, torch.float16, "cuda", layout="vllm", seed=2)
    q = torch.randn(n, hkv * group, d, device="cuda", dtype=torch.float16)
    k, v = fp8_caches(kv, "vllm", KS, VS)
    fitted, plan = _call(q, kv, k, v, 0, False, True)
    assert plan["fit_min_partition"] == 512
    assert _predicted(lens, hkv, plan, _gran(True, d)) == plan["partition_size"]
    fixed, _ = _call(q, kv, k, v, plan["partition_size"], False, True)
    assert torch.equal(fitted, fixed)
    assert_attention_close(fitted, oracle_dense_fp8(q, kv, k, v, KS, VS), torch.float16, "planned size kept")


def test_graph_replay_refits_to_each_batch():
    # One capture; each replay reads new lengths (within the captured bound)
    # from device memory and must fit its own size.
    n, hkv, group, d = 96, 1, 8, 256
    full = _lognormal_lens(n, seed=11, median=6000)
    kv = make_paged_kv(full, hkv, d, 32, torch.bfloat16, "cuda", seed=3)
    k, v = fp8_caches(kv, "nhd", KS, VS)
    q = torch.randn(n, hkv * group, d, device="cuda", dtype=torch.bfloat16)
    out = torch.full_like(q, float("nan"))
    ws = alloc_ws(n, hkv * group, d, capi.num_partitions(n, hkv, d, 32, MAX_LEN), q.device)

    def step():
        capi.decode(q, k, v, kv.block_tables, kv.seq_lens, d**-0.5, MAX_LEN, out, ws, k_scale=KS, v_scale=VS)

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        step()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    plan = capi.plan(q, k, v, kv.block_tables, kv.seq_lens, d**-0.5, MAX_LEN, out, ws, k_scale=KS, v_scale=VS)
    assert plan["fit_min_partition"] == 512
    chosen = set()
    for scale in (1.0, 0.5, 0.2):
        lens = [int(l * scale) if i % 9 else 0 for i, l in enumerate(full)]  # within what the cache holds
        kv.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
        q.normal_()
        graph.replay()
        torch.cuda.synchronize()
        ps = _predicted(lens, hkv, plan, _gran(True, d))
        chosen.add(ps)
        fixed, _ = _call(q, kv, k, v, ps, False, True)
        assert torch.equal(out, fixed), f"replay at lengths x{scale} did not use partition_size={ps}"
        assert_attention_close(out, oracle_dense_fp8(q, kv, k, v, KS, VS), torch.bfloat16, f"graph replay x{scale}")
    assert len(chosen) > 1, chosen  # the batches really asked for different sizes
    del graph
