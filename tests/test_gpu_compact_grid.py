"""GPU: the compact grid -- live (sequence, KV head, partition) items numbered
densely, CTA b running items b, b + G, ... -- gives bit-identical results to
the dense grid (one CTA per possible partition), and with DK_FLAG_PERSISTENT
(one wave of CTAs) every CTA runs several items in a row, carrying its ring
and barrier phases from item to item.  Cases: skewed lengths with empty
sequences, 16-bit and e4m3 caches, head_dim 128 and 256, the merge kernel,
the single-launch merge and the single pass."""

import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import capi
from decodekernels_b200.testing import make_paged_kv
from gpu_helpers import assert_attention_close, fp8_caches, oracle_dense, oracle_dense_fp8, run_capi

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

KS, VS = 0.02, 0.015


def _lens(n, seed, max_len=4096):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (n,), generator=g)
    lens[::7] = 0  # empty sequences
    lens[1] = max_len
    return lens.tolist()


def _q(n, hq, d, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(n, hq, d, generator=g, device="cuda", dtype=torch.float32).to(dtype)


def _run(q, kv, ps, flags, counters, k8=None, v8=None):
    if k8 is None:
        out, _, plan = run_capi(q, kv, partition_size=ps, flags=flags, counters=counters)
        return out, plan

    n, hq, d = q.shape
    L = int(kv.seq_lens.max().item())
    parts = -(-L // ps)
    ws = tuple(torch.full(s, float("nan"), device="cuda") for s in ((n, hq, parts, d), (n, hq, parts), (n, hq, parts)))
    if counters:
        ws = (*ws, torch.zeros(n * k8.shape[2], dtype=torch.int32, device="cuda"))
    out = torch.full_like(q, float("nan"))
    plan = capi.plan(q, k8, v8, kv.block_tables, kv.seq_lens, d**-0.5, L, out, ws, ps, False, flags, KS, VS)
    capi.decode(q, k8, v8, kv.block_tables, kv.seq_lens, d**-0.5, L, out, ws, ps, False, flags=flags, k_scale=KS,
                v_scale=VS)
    torch.cuda.synchronize()
    return out, plan


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("dtype,d,group,layout,bs", [(torch.float16, 128, 8, "vllm", 16),
                                                     (torch.bfloat16, 128, 4, "hnd", 16),
                                                     (torch.bfloat16, 256, 8, "nhd", 32)])
@pytest.mark.parametrize("merge", ["kernel", "fused"])
@pytest.mark.parametrize("ps", [64, 512])
def test_persistent_matches_default_grid(fp8, dtype, d, group, layout, bs, merge, ps):
    # 48 sequences x 2 KV heads; at 64-token partitions ~3000 items, several
    # per CTA of one wave (the default grid is compact too: 64 partitions),
    # at 512 the default grid is the dense one (8 partitions)
    lens = _lens(48, seed=d + group)
    kv = make_paged_kv(lens, 2, d, bs, dtype, "cuda", layout=layout, seed=d)
    q = _q(len(lens), 2 * group, d, dtype, seed=group)
    k8 = v8 = None
    if fp8:
        k8, v8 = fp8_caches(kv, layout, KS, VS)
    counters = merge == "fused"
    flags = capi.DK_FLAG_FORCE_FUSED_MERGE if counters else 0
    default, plan = _run(q, kv, ps, flags, counters, k8, v8)
    assert plan["path"] == capi.DK_PATH_TMA_MMA and plan["num_partitions"] == 4096 // ps
    compact, _ = _run(q, kv, ps, flags | capi.DK_FLAG_PERSISTENT, counters, k8, v8)
    assert torch.equal(compact, default), "persistent grid differs from the default grid"
    want = oracle_dense_fp8(q, kv, k8, v8, KS, VS) if fp8 else oracle_dense(q, kv)
    assert_attention_close(compact, want, dtype, "persistent")


@pytest.mark.parametrize("d", [128, 256])
def test_persistent_single_pass_writes_zeros(d):
    lens = [0, 5, 0, 300, 64, 0, 1]
    kv = make_paged_kv(lens, 1, d, 16, torch.float16, "cuda", seed=3)
    q = _q(len(lens), 8, d, torch.float16, seed=4)
    out, _, plan = run_capi(q, kv, workspace=None, flags=capi.DK_FLAG_PERSISTENT)
    assert plan["split"] == 0
    want = oracle_dense(q, kv)
    assert_attention_close(out, want, torch.float16, "persistent single pass")
    assert (out[[0, 2, 5]] == 0).all()


def test_persistent_repeated_calls_identical():
    lens = _lens(64, seed=11, max_len=6000)
    kv = make_paged_kv(lens, 2, 128, 16, torch.bfloat16, "cuda", seed=5)
    q = _q(len(lens), 16, 128, torch.bfloat16, seed=6)
    first, _ = _run(q, kv, 64, capi.DK_FLAG_PERSISTENT, False)
    for _ in range(10):
        again, _ = _run(q, kv, 64, capi.DK_FLAG_PERSISTENT, False)
        assert torch.equal(again, first)
    assert capi.wait_timeouts(0) == 0


@pytest.mark.parametrize("n", [128, 129, 512, 513])
def test_compact_grid_at_its_sequence_limit(n):
    """128 sequences: the small compact instance's largest batch (4 lengths
    per lane); 129 takes the large one; 512: its largest batch (16 lengths
    per lane); 513 falls back to the dense grid.  All agree bit for bit with
    the dense grid and match the oracle on a sample of sequences."""
    g = torch.Generator().manual_seed(n)
    lens = torch.randint(0, 1200, (n,), generator=g).tolist()
    kv = make_paged_kv(lens, 1, 128, 16, torch.bfloat16, "cuda", layout="nhd", seed=n)
    q = _q(n, 4, 128, torch.bfloat16, seed=n)
    default, plan = _run(q, kv, 64, 0, False)
    persistent, _ = _run(q, kv, 64, capi.DK_FLAG_PERSISTENT, False)
    assert torch.equal(persistent, default)
    want = oracle_dense(q[:64], type(kv)(kv.k_cache, kv.v_cache, kv.block_tables[:64], kv.seq_lens[:64],
                                         kv.block_size))
    assert_attention_close(default[:64], want, torch.bfloat16, f"n={n}")


@pytest.mark.parametrize("fp8", [False, True])
def test_persistent_lse_partials(fp8):
    """The LSE-partials entry point (sequence sharding) on the persistent grid
    writes the same rows as on the default grid."""
    lens = _lens(24, seed=5, max_len=3000)
    kv = make_paged_kv(lens, 2, 128, 16, torch.float16, "cuda", layout="hnd", seed=6)
    q = _q(len(lens), 8, 128, torch.float16, seed=7)
    k, v, ks, vs = kv.k_cache, kv.v_cache, 1.0, 1.0
    if fp8:
        k, v = fp8_caches(kv, "hnd", KS, VS)
        ks, vs = KS, VS
    n, hq, d = q.shape
    L = max(lens)
    rows = []
    for flags in (0, capi.DK_FLAG_PERSISTENT):
        part = torch.full((n, hq, d + 4), float("nan"), device="cuda")
        ws = tuple(torch.empty(s, device="cuda") for s in ((n, hq, 64, d), (n, hq, 64), (n, hq, 64)))
        capi.decode_lse(q, k, v, kv.block_tables, kv.seq_lens, d**-0.5, L, part, ws, 64, flags=flags, k_scale=ks,
                        v_scale=vs)
        torch.cuda.synchronize()
        rows.append(part)
    assert torch.equal(rows[0][..., :d + 1], rows[1][..., :d + 1])
