"""GPU parity: the sm_100a kernels against the CPU oracle and the golden
vectors of the reference, through the C ABI (libdk_b200.so) and through the
drop-in torch op.

Shapes follow the reference's own GPU tests (DecodeKernels
tests/test_kernels.py:36-144) plus the cases this implementation adds
(per-shape partition sizes, the CUDA-core path, block sizes that use several
TMA boxes per page or one box per several tiles, workspace indexing).
"""

import numpy as np
import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import capi
from decodekernels_b200.testing import make_paged_kv
from golden_cases import build, load_cases, outputs
from gpu_helpers import (ATTN_TOL, alloc_ws, assert_attention_close, assert_workspace_matches, oracle_dense,
                         run_capi)

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

DTYPES = [torch.float16, torch.bfloat16]
HALF_CASES = [c for c in load_cases() if c["dtype"] != "float32"]


def _q(num_seqs, num_q_heads, head_dim, dtype, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(num_seqs, num_q_heads, head_dim, generator=g, device="cuda", dtype=dtype)


# ---------------------------------------------------------------------------
# Golden vectors of the reference
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", HALF_CASES, ids=[c["name"] for c in HALF_CASES])
@pytest.mark.parametrize("path", ["planner", "simt"])
def test_golden_cases(case, path):
    q, kv = build(case, "cuda")
    gold = outputs(case)
    out, _, plan = run_capi(q, kv, scale=case["scale"], force_simt=path == "simt")
    if path == "planner" and case["block_size"] >= 8:
        assert plan["path"] == capi.DK_PATH_TMA_MMA, plan
    dtype = q.dtype
    # against the reference's dense output (rounded to the dtype) and its fp32 split-K merge
    assert_attention_close(out, gold["dense"], dtype, f"{case['name']} vs reference dense")
    assert_attention_close(out, gold["split_512"], dtype, f"{case['name']} vs reference split-K")


@pytest.mark.parametrize("case", HALF_CASES, ids=[c["name"] for c in HALF_CASES])
def test_golden_workspace_indexing(case):
    """With the reference's 512-token (and each golden case's other) partition
    size, every live workspace row matches the oracle's partition statistics
    and no row past a sequence's end is written."""
    q, kv = build(case, "cuda")
    gold = outputs(case)
    max_len = max(case["seq_lens"])
    for ps in sorted(set(case["partitions"]) | {64}):
        if -(-max_len // ps) < 2:
            continue  # single pass: no workspace
        out, ws, plan = run_capi(q, kv, scale=case["scale"], partition_size=ps)
        assert plan["split"] == 1 and plan["partition_size"] == ps
        assert_workspace_matches(ws, kv, q, ps, scale=case["scale"], what=f"{case['name']} ps={ps}")
        assert_attention_close(out, gold["dense"], q.dtype, f"{case['name']} ps={ps}")


# ---------------------------------------------------------------------------
# The reference's GPU test matrix (tests/test_kernels.py:36-98)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("group", [1, 4, 8])
@pytest.mark.parametrize("block_size", [16, 32])
def test_paged_attention_short(dtype, head_dim, group, block_size):
    seq_lens = [1, 2, 17, 100, 255, 512]
    kv = make_paged_kv(seq_lens, 2, head_dim, block_size, dtype, "cuda")
    q = _q(len(seq_lens), 2 * group, head_dim, dtype)
    out = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    assert_attention_close(out, oracle_dense(q, kv), dtype, "short")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("group", [1, 8])
def test_paged_attention_split_k(dtype, head_dim, group):
    seq_lens = [1, 511, 512, 513, 1024, 1025, 3000, 8192]
    kv = make_paged_kv(seq_lens, 2, head_dim, 16, dtype, "cuda")
    q = _q(len(seq_lens), 2 * group, head_dim, dtype)
    out = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    assert_attention_close(out, oracle_dense(q, kv), dtype, "split")


@pytest.mark.parametrize("layout", ["hnd", "vllm"])
@pytest.mark.parametrize("seq_lens", [[5, 300], [700, 2000]])
def test_paged_attention_strided_layouts(layout, seq_lens):
    dtype = torch.float16
    kv = make_paged_kv(seq_lens, 2, 128, 16, dtype, "cuda", layout=layout)
    assert not kv.k_cache.is_contiguous()
    q = _q(len(seq_lens), 8, 128, dtype)
    out = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    assert_attention_close(out, oracle_dense(q, kv), dtype, layout)


@pytest.mark.parametrize("max_seq_len", [100, 2000])
def test_paged_attention_empty_sequences(max_seq_len):
    seq_lens = [0, 50, 0, max_seq_len]
    kv = make_paged_kv(seq_lens, 2, 64, 16, torch.float16, "cuda")
    q = _q(len(seq_lens), 4, 64, torch.float16)
    out = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    assert torch.isfinite(out).all()
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0
    assert_attention_close(out, oracle_dense(q, kv), torch.float16, "empty")


def test_paged_attention_custom_scale_and_output_buffer():
    kv = make_paged_kv([64, 900], 1, 128, 16, torch.bfloat16, "cuda")
    q = _q(2, 4, 128, torch.bfloat16)
    out = torch.full_like(q, float("nan"))
    dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale=0.05, out=out)
    assert_attention_close(out, oracle_dense(q, kv, scale=0.05), torch.bfloat16, "scale")


def test_paged_attention_cuda_graph_replay():
    """Preallocated buffers make the op capturable; replay tracks new cache
    contents and lengths within the captured max_seq_len (tests/test_kernels.py:101-133)."""
    dtype = torch.float16
    max_seq_len = 2048
    kv = make_paged_kv([max_seq_len] * 3, 2, 128, 16, dtype, "cuda")
    kv.seq_lens.copy_(torch.tensor([300, 1500, 40], dtype=torch.int32))
    q = _q(3, 8, 128, dtype)
    out = torch.empty_like(q)
    ws = dk.alloc_workspace(3, 8, 128, max_seq_len, "cuda")

    def step():
        dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=max_seq_len,
                                  out=out, workspace=ws)

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        step()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for new_lens in ([300, 1500, 40], [2048, 1, 777], [0, 2048, 513]):
        kv.seq_lens.copy_(torch.tensor(new_lens, dtype=torch.int32))
        q.normal_()
        graph.replay()
        torch.cuda.synchronize()
        assert_attention_close(out, oracle_dense(q, kv), dtype, f"graph {new_lens}")
    del graph


def test_paged_attention_rejects_bad_inputs():
    kv = make_paged_kv([10], 2, 128, 16, torch.float16, "cuda")
    q = _q(1, 32, 128, torch.float16)  # group 16 > 8
    with pytest.raises(RuntimeError, match="GQA group"):
        dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    kv96 = make_paged_kv([10], 2, 96, 16, torch.float16, "cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        dk.paged_attention_decode(_q(1, 2, 96, torch.float16), kv96.k_cache, kv96.v_cache, kv96.block_tables,
                                  kv96.seq_lens)
    kv2 = make_paged_kv([1000], 2, 128, 16, torch.float16, "cuda")
    q2 = _q(1, 4, 128, torch.float16)
    empty = torch.empty(0, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="tmp_out must be"):
        dk.paged_attention_decode(q2, kv2.k_cache, kv2.v_cache, kv2.block_tables, kv2.seq_lens, max_seq_len=1000,
                                  workspace=(empty, empty, empty))
    with pytest.raises(RuntimeError, match="GQA group"):
        capi.decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, 0.1, 10, torch.empty_like(q))


# ---------------------------------------------------------------------------
# Beyond the reference's matrix
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("block_size", [8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("dtype", DTYPES)
def test_block_sizes_tma_path(block_size, dtype):
    """Pages smaller than a tile (several boxes per tile) and larger (several tiles per page)."""
    seq_lens = [1, 63, 64, 65, 700, 1500]
    kv = make_paged_kv(seq_lens, 2, 128, block_size, dtype, "cuda", seed=block_size)
    q = _q(len(seq_lens), 8, 128, dtype, seed=block_size)
    for ps in (0, 64, 512):
        out, _, plan = run_capi(q, kv, partition_size=ps)
        assert plan["path"] == capi.DK_PATH_TMA_MMA
        assert_attention_close(out, oracle_dense(q, kv), dtype, f"bs={block_size} ps={ps}")


@pytest.mark.parametrize("block_size", [1, 3, 12, 48])
def test_block_sizes_simt_path(block_size):
    """Block sizes the 64-token TMA tile cannot use go to the CUDA-core path."""
    seq_lens = [1, 37, 200, 600]
    kv = make_paged_kv(seq_lens, 2, 64, block_size, torch.bfloat16, "cuda", seed=block_size)
    q = _q(len(seq_lens), 8, 64, torch.bfloat16)
    out, _, plan = run_capi(q, kv)
    assert plan["path"] == capi.DK_PATH_SIMT
    assert_attention_close(out, oracle_dense(q, kv), torch.bfloat16, f"bs={block_size}")


def test_unaligned_cache_uses_simt_path():
    """Strides that are multiples of head_dim / 32 but not of 16 bytes (accepted by the reference)."""
    d = 128
    base = torch.randn(40, 16, 2, d + 4, dtype=torch.float16, device="cuda")  # row stride d+4 elements = 264 B
    k = base[..., :d]
    v = torch.randn(40, 16, 2, d + 4, dtype=torch.float16, device="cuda")[..., 4:]
    seq_lens = torch.tensor([100, 300], dtype=torch.int32, device="cuda")
    g = torch.Generator().manual_seed(3)
    tables = torch.randperm(40, generator=g)[:38].view(2, 19).to(torch.int32).cuda()
    from decodekernels_b200.testing import PagedKV

    kv = PagedKV(k, v, tables, seq_lens, 16)
    q = _q(2, 8, d, torch.float16)
    out, _, plan = run_capi(q, kv)
    assert plan["path"] == capi.DK_PATH_SIMT
    assert_attention_close(out, oracle_dense(q, kv), torch.float16, "unaligned")


@pytest.mark.parametrize("dtype", DTYPES)
def test_garbage_in_unused_slots_and_table_entries(dtype):
    """NaN in the unused tail of a sequence's last page and garbage block ids
    past its end must not reach the output."""
    seq_lens = [5, 70, 1000]
    kv = make_paged_kv(seq_lens, 2, 128, 16, dtype, "cuda", extra_blocks=8)
    bs = 16
    for s, L in enumerate(seq_lens):
        nb = -(-L // bs)
        last = int(kv.block_tables[s, nb - 1])
        if L % bs:
            kv.k_cache[last, L % bs:] = float("nan")
            kv.v_cache[last, L % bs:] = float("nan")
        if nb < kv.block_tables.shape[1]:
            kv.block_tables[s, nb:] = 2**30
    q = _q(len(seq_lens), 8, 128, dtype)
    ref = oracle_dense(q, kv)
    for ps in (0, 64):
        out, _, _ = run_capi(q, kv, partition_size=ps)
        assert_attention_close(out, ref, dtype, f"garbage ps={ps}")
    out, _, _ = run_capi(q, kv, force_simt=True)
    assert_attention_close(out, ref, dtype, "garbage simt")


@pytest.mark.parametrize("head_dim", [64, 128, 256])
def test_partition_sizes_agree(head_dim):
    """Every partition size (and the single pass) gives the same answer."""
    seq_lens = [1, 513, 4100, 64, 2000]
    kv = make_paged_kv(seq_lens, 2, head_dim, 16, torch.bfloat16, "cuda")
    q = _q(len(seq_lens), 16, head_dim, torch.bfloat16)
    ref = oracle_dense(q, kv)
    for ps in (64, 128, 512, 4096):
        out, ws, plan = run_capi(q, kv, partition_size=ps)
        assert_attention_close(out, ref, torch.bfloat16, f"D={head_dim} ps={ps}")
    out, _, plan = run_capi(q, kv, workspace=None)
    assert plan["split"] == 0
    assert_attention_close(out, ref, torch.bfloat16, f"D={head_dim} single pass")


def test_max_seq_len_below_actual_clamps_like_reference():
    """A too-small max_seq_len never reads out of bounds: lengths above it
    count as max_seq_len on every path, so no block-table entry at or past
    ceil(max_seq_len / block_size) is read.  (The reference's partition
    kernel takes its 512-token partition up to seq_len there, reading past
    a block table sized for max_seq_len.)"""
    kv = make_paged_kv([300], 1, 64, 16, torch.float16, "cuda")
    q = _q(1, 4, 64, torch.float16)
    for kwargs in ({"workspace": None}, {"partition_size": 64}, {}, {"force_simt": True}):
        out, _, plan = run_capi(q, kv, max_seq_len=100, **kwargs)
        kv.seq_lens.fill_(100)
        assert_attention_close(out, oracle_dense(q, kv), torch.float16, f"clamped {kwargs}")
        kv.seq_lens.fill_(300)


def test_no_wait_timeouts():
    """No bounded device wait gave up during this session."""
    assert capi.wait_timeouts(0) == 0


# ---------------------------------------------------------------------------
# Planner: mixed lengths, workspace capacity, batch sizes
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("head_dim,group,layout", [(128, 8, "vllm"), (128, 4, "hnd"), (64, 1, "nhd"), (256, 8, "nhd")])
def test_planner_varied_lengths(dtype, head_dim, group, layout):
    """Mixed lengths with empty sequences and one long one, at the planner's
    partition size and at the smallest (one tile per partition)."""
    g = torch.Generator().manual_seed(head_dim + group)
    lens = torch.randint(1, 3000, (37,), generator=g).tolist()
    lens[3] = lens[20] = 0
    lens[7] = 9000
    kv = make_paged_kv(lens, 2, head_dim, 16, dtype, "cuda", layout=layout, seed=group)
    q = _q(len(lens), 2 * group, head_dim, dtype, seed=head_dim)
    for ps in (0, 64):
        out, _, plan = run_capi(q, kv, partition_size=ps)
        assert plan["path"] == capi.DK_PATH_TMA_MMA and plan["split"] == 1
        out_np = out.float().cpu()
        assert torch.count_nonzero(out_np[3]) == 0 and torch.count_nonzero(out_np[20]) == 0
        assert_attention_close(out, oracle_dense(q, kv), dtype, f"varied ps={ps}")


@pytest.mark.parametrize("rows", [2, 3, 5])
def test_planner_small_workspace_grows_partitions(rows):
    """A workspace with fewer rows than the planner wants: partitions grow
    so ceil(max_seq_len / partition_size) fits."""
    lens = [20000, 5, 3000, 64]
    kv = make_paged_kv(lens, 2, 128, 16, torch.bfloat16, "cuda", seed=rows)
    q = _q(len(lens), 16, 128, torch.bfloat16)
    ws = alloc_ws(len(lens), 16, 128, rows, q.device)
    out, _, plan = run_capi(q, kv, workspace=ws)
    assert plan["path"] == capi.DK_PATH_TMA_MMA and plan["num_partitions"] <= rows
    assert plan["num_partitions"] * plan["partition_size"] >= 20000
    assert_attention_close(out, oracle_dense(q, kv), torch.bfloat16, f"{rows} rows")


def test_planner_matches_fixed_partitions():
    """The planner's split and the reference's 512-token split agree to
    fp32 rounding (same math, different partition boundaries)."""
    lens = [1, 63, 64, 65, 511, 512, 513, 4000, 12000, 0, 777]
    kv = make_paged_kv(lens, 4, 128, 32, torch.float16, "cuda", layout="vllm", seed=5)
    q = _q(len(lens), 32, 128, torch.float16)
    a, _, pa = run_capi(q, kv)
    b, _, pb = run_capi(q, kv, partition_size=512)
    assert pa["path"] == pb["path"] == capi.DK_PATH_TMA_MMA
    assert (a.float() - b.float()).abs().max().item() <= 2e-3


@pytest.mark.parametrize("n", [1024, 4099])
def test_planner_large_batches(n):
    g = torch.Generator().manual_seed(n)
    lens = torch.randint(0, 200, (n,), generator=g).tolist()
    kv = make_paged_kv(lens, 1, 64, 16, torch.bfloat16, "cuda", seed=n)
    q = _q(n, 4, 64, torch.bfloat16)
    out, _, plan = run_capi(q, kv)
    assert plan["path"] == capi.DK_PATH_TMA_MMA
    assert_attention_close(out, oracle_dense(q, kv), torch.bfloat16, f"n={n}")
