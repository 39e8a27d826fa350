"""GPU: decode over e4m3 (FP8) KV caches -- the TMA path (head_dim 128 / 256,
conversion in registers) and the CUDA-core path (head_dim 64, unaligned
layouts) -- against the oracle on the dequantised caches (code * scale),
with the same tolerance as 16-bit caches; through the C ABI, the torch op,
the single-launch merge and the LSE partials; and end to end with caches
written by reshape_and_cache."""

import numpy as np
import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import capi
from decodekernels_b200.testing import make_paged_kv
from gpu_helpers import assert_attention_close, fp8_caches, oracle_dense_fp8, run_capi
from oracle import sharded_lse as sl

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

KS, VS = 0.02, 0.015  # values ~ N(0, 1) -> codes of magnitude ~50-70, inside e4m3's range


def _q(n, hq, d, dtype, seed=1, mag=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(n, hq, d, generator=g, device="cuda", dtype=torch.float32) * mag).to(dtype)


def _case(dtype, d, group, layout, bs=16, seed=0, lens=(1, 0, 63, 64, 65, 700, 2500, 17, 4096)):
    kv = make_paged_kv(list(lens), 2, d, bs, dtype, "cuda", layout=layout, seed=seed + d)
    q = _q(len(lens), 2 * group, d, dtype, seed=seed + group)
    k8, v8 = fp8_caches(kv, layout, KS, VS)
    want = oracle_dense_fp8(q, kv, k8, v8, KS, VS)
    return kv, q, k8, v8, want


def _run(q, kv, k8, v8, **kw):
    class KV8:
        k_cache, v_cache, block_tables, seq_lens = k8, v8, kv.block_tables, kv.seq_lens

    kw.setdefault("flags", 0)
    n, hq, d = q.shape
    out = torch.full_like(q, float("nan"))
    L = int(kv.seq_lens.max().item())
    ws = kw.pop("workspace", "auto")
    ps = kw.pop("partition_size", 0)
    if ws == "auto":
        parts = -(-L // ps) if ps else capi.num_partitions(n, k8.shape[2], d, k8.shape[1], L)
        ws = tuple(torch.empty(s, device="cuda") for s in ((n, hq, parts, d), (n, hq, parts), (n, hq, parts)))
        if kw.pop("counters", False):
            ws = (*ws, torch.zeros(n * k8.shape[2], dtype=torch.int32, device="cuda"))
    plan = capi.plan(q, k8, v8, kv.block_tables, kv.seq_lens, d**-0.5, L, out, ws, ps, kw.get("force_simt", False),
                     kw["flags"], KS, VS)
    capi.decode(q, k8, v8, kv.block_tables, kv.seq_lens, d**-0.5, L, out, ws, ps, kw.get("force_simt", False),
                flags=kw["flags"], k_scale=KS, v_scale=VS)
    torch.cuda.synchronize()
    return out, plan


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d,group,layout", [(128, 8, "vllm"), (128, 4, "hnd"), (256, 8, "nhd"), (256, 1, "vllm"),
                                            (64, 8, "nhd"), (64, 4, "vllm")])
@pytest.mark.parametrize("path", ["planner", "single", "ps64", "simt", "fused"])
def test_fp8_matches_oracle(dtype, d, group, layout, path):
    kv, q, k8, v8, want = _case(dtype, d, group, layout)
    kw = {}
    if path == "single":
        kw["workspace"] = None
    elif path == "ps64":
        kw["partition_size"] = 64
    elif path == "simt":
        kw["force_simt"] = True
    elif path == "fused":
        kw.update(counters=True, flags=capi.DK_FLAG_FORCE_FUSED_MERGE)
    out, plan = _run(q, kv, k8, v8, **kw)
    expect_tma = d >= 128 and path != "simt"
    assert plan["path"] == (capi.DK_PATH_TMA_MMA if expect_tma else capi.DK_PATH_SIMT), plan
    out_np = out.float().cpu()
    assert torch.count_nonzero(out_np[1]) == 0
    assert_attention_close(out, want, dtype, f"fp8 {path} D{d} g{group} {layout}")


@pytest.mark.parametrize("bs", [8, 32, 64, 128])
def test_fp8_block_sizes(bs):
    kv, q, k8, v8, want = _case(torch.bfloat16, 128, 8, "nhd", bs=bs, seed=bs)
    out, plan = _run(q, kv, k8, v8)
    assert plan["path"] == capi.DK_PATH_TMA_MMA
    assert_attention_close(out, want, torch.bfloat16, f"fp8 bs={bs}")


def test_fp8_large_bf16_queries_are_prescaled_exactly():
    """bf16 queries far outside f16's range (|q| ~ 1e5) run through the f16
    mma after an exact power-of-two prescale."""
    kv, _, k8, v8, _ = _case(torch.bfloat16, 128, 8, "vllm", lens=(300, 2000, 5))
    q = _q(3, 16, 128, torch.bfloat16, seed=5, mag=1e5)
    want = oracle_dense_fp8(q, kv, k8, v8, KS, VS)
    out, _ = _run(q, kv, k8, v8)
    assert torch.isfinite(out).all()
    assert_attention_close(out, want, torch.bfloat16, "large q")


def test_fp8_torch_op_and_lse():
    kv, q, k8, v8, want = _case(torch.float16, 128, 4, "hnd", lens=(0, 3000, 40, 513))
    out = dk.paged_attention_decode(q, k8, v8, kv.block_tables, kv.seq_lens, k_scale=KS, v_scale=VS)
    torch.cuda.synchronize()
    assert_attention_close(out, want, torch.float16, "torch op")
    ws = dk.alloc_workspace(4, 8, 128, 3000, "cuda", num_kv_heads=2, merge_counters=True)
    out2 = dk.paged_attention_decode(q, k8.view(torch.float8_e4m3fn), v8.view(torch.float8_e4m3fn), kv.block_tables,
                                     kv.seq_lens, max_seq_len=3000, workspace=ws, k_scale=KS, v_scale=VS)
    torch.cuda.synchronize()
    assert_attention_close(out2, want, torch.float16, "torch op, float8 dtype, counters")
    part = dk.paged_attention_decode_lse(q, k8, v8, kv.block_tables, kv.seq_lens, k_scale=KS, v_scale=VS)
    torch.cuda.synchronize()
    from oracle import cache_write as cw

    kd = cw.e4m3_decode(k8.cpu().numpy()) * np.float32(KS)
    vd = cw.e4m3_decode(v8.cpu().numpy()) * np.float32(VS)
    _, lse_want = sl.attention_lse(q.cpu(), kd, vd, kv.block_tables.cpu().numpy(), kv.seq_lens.cpu().numpy())
    got = part.cpu().numpy()
    fin = np.isfinite(lse_want)
    np.testing.assert_allclose(got[..., 128][fin], lse_want[fin], atol=2e-3, rtol=1e-4)
    assert_attention_close(torch.from_numpy(got[..., :128]).to(torch.float16), want, torch.float16, "lse o")


def test_fp8_written_by_reshape_and_cache():
    """Tokens written into an e4m3 cache by reshape_and_cache decode like the
    oracle on that cache (the two steps of a serving iteration)."""
    dtype, lens = torch.bfloat16, [1, 300, 77, 1024]
    kv = make_paged_kv(lens, 2, 128, 16, dtype, "cuda", layout="nhd", seed=3)
    nb = kv.k_cache.shape[0]
    k8 = torch.zeros(nb, 16, 2, 128, dtype=torch.uint8, device="cuda")
    v8 = torch.zeros_like(k8)
    bt = kv.block_tables.cpu()
    slots, keys, values = [], [], []
    for s, L in enumerate(lens):
        for t in range(L):
            b = int(bt[s, t // 16])
            slots.append(b * 16 + t % 16)
            keys.append(kv.k_cache[b, t % 16])
            values.append(kv.v_cache[b, t % 16])
    dk.reshape_and_cache(torch.stack(keys), torch.stack(values), k8, v8,
                         torch.tensor(slots, dtype=torch.int64, device="cuda"), KS, VS)
    q = _q(len(lens), 16, 128, dtype)
    out = dk.paged_attention_decode(q, k8, v8, kv.block_tables, kv.seq_lens, k_scale=KS, v_scale=VS)
    torch.cuda.synchronize()
    assert_attention_close(out, oracle_dense_fp8(q, kv, k8, v8, KS, VS), dtype, "written fp8 cache")
