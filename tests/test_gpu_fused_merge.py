"""GPU: the single-launch merge (merge counters in the workspace).  The last
partition of each (sequence, KV head) to finish merges that pair's
partitions; results match the oracle and the two-launch path, the counters
return to zero after every call, and the call is one kernel launch."""

import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import capi
from decodekernels_b200.testing import make_paged_kv
from golden_cases import build, load_cases, outputs
from gpu_helpers import assert_attention_close, oracle_dense, run_capi

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

HALF_CASES = [c for c in load_cases() if c["dtype"] != "float32"]


def _q(n, hq, d, dtype, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(n, hq, d, generator=g, device="cuda", dtype=dtype)


@pytest.mark.parametrize("case", HALF_CASES, ids=[c["name"] for c in HALF_CASES])
@pytest.mark.parametrize("ps", [0, 64, 512])
def test_golden_cases_single_launch(case, ps):
    q, kv = build(case, "cuda")
    gold = outputs(case)
    out, ws, plan = run_capi(q, kv, scale=case["scale"], partition_size=ps, counters=True,
                             flags=capi.DK_FLAG_FORCE_FUSED_MERGE)
    if plan["split"]:
        assert plan["launches"] == 1
    assert_attention_close(out, gold["dense"], q.dtype, f"{case['name']} ps={ps}")
    assert int(ws[3].abs().sum().item()) == 0, "merge counters not reset"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim,group,layout,bs", [(128, 8, "vllm", 16), (64, 1, "nhd", 32), (256, 8, "nhd", 32),
                                                      (128, 4, "hnd", 8)])
@pytest.mark.parametrize("simt", [False, True])
def test_varied_lengths_match_two_launch(dtype, head_dim, group, layout, bs, simt):
    g = torch.Generator().manual_seed(head_dim + group)
    lens = torch.randint(1, 3000, (29,), generator=g).tolist()
    lens[2] = lens[11] = 0
    lens[5] = 7000
    kv = make_paged_kv(lens, 2, head_dim, bs, dtype, "cuda", layout=layout, seed=group)
    q = _q(len(lens), 2 * group, head_dim, dtype, seed=head_dim)
    want = oracle_dense(q, kv)
    for ps in (0, 64):
        a, ws, pa = run_capi(q, kv, partition_size=ps, force_simt=simt, counters=True,
                             flags=capi.DK_FLAG_FORCE_FUSED_MERGE)
        b, _, pb = run_capi(q, kv, partition_size=ps, force_simt=simt)
        assert pa["split"] == 1 and pa["launches"] == 1 and pb["launches"] == 2
        assert torch.count_nonzero(a[2]) == 0 and torch.count_nonzero(a[11]) == 0
        assert_attention_close(a, want, dtype, f"fused ps={ps} simt={simt}")
        assert (a.float() - b.float()).abs().max().item() <= 4e-3
        assert int(ws[3].abs().sum().item()) == 0


def test_repeated_calls_and_graph_replay():
    """Counters left at zero make back-to-back calls and graph replays correct
    (the drop-in torch op with a 4-tuple workspace)."""
    dtype = torch.float16
    n, hq, hkv, L = 16, 8, 2, 2048  # one wave of small merges: the planner takes the single launch
    kv = make_paged_kv([L] * n, hkv, 128, 16, dtype, "cuda", layout="vllm")
    q = _q(n, hq, 128, dtype)
    out = torch.empty_like(q)
    ws = dk.alloc_workspace(n, hq, 128, L, "cuda", num_kv_heads=hkv, merge_counters=True)
    assert len(ws) == 4
    plan = capi.plan(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, 128**-0.5, L, out, ws)
    assert plan["split"] == 1 and plan["launches"] == 1

    def step():
        dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=L, out=out,
                                  workspace=ws)

    g = torch.Generator().manual_seed(3)
    for _ in range(2):
        lens = torch.randint(0, L + 1, (n,), generator=g, dtype=torch.int32)
        kv.seq_lens.copy_(lens)
        step()
        step()
        torch.cuda.synchronize()
        assert_attention_close(out, oracle_dense(q, kv), dtype, "eager")
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        step()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        kv.seq_lens.copy_(torch.randint(0, L + 1, (n,), generator=g, dtype=torch.int32))
        q.normal_()
        graph.replay()
        torch.cuda.synchronize()
        assert_attention_close(out, oracle_dense(q, kv), dtype, "graph")
    del graph
    assert int(ws[3].abs().sum().item()) == 0


def test_merge_size_decides_without_the_flag():
    """Without the flag, counters are used only when a pair's rows are small."""
    kv = make_paged_kv([600, 5000], 2, 128, 16, torch.float16, "cuda")
    q = _q(2, 16, 128, torch.float16)
    _, _, small = run_capi(q, kv, partition_size=512, counters=True)  # 10 rows x 8 heads x 130 floats
    _, _, big = run_capi(q, kv, partition_size=64, counters=True)  # 79 rows
    assert small["split"] == big["split"] == 1
    assert small["launches"] == 1 and big["launches"] == 2


def test_torch_op_validates_counters():
    kv = make_paged_kv([1000], 2, 128, 16, torch.float16, "cuda")
    q = _q(1, 8, 128, torch.float16)
    tmp, ml, es = dk.alloc_workspace(1, 8, 128, 1000, "cuda", num_kv_heads=2)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")  # needs num_seqs * num_kv_heads = 2
    with pytest.raises(RuntimeError, match="merge_counters"):
        dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=1000,
                                  workspace=(tmp, ml, es, bad))
