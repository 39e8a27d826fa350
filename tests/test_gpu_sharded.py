"""GPU: KV-head sharding with the real kernels.

* On one GPU: every rank's shard (strided views of one cache) is computed
  with the sm_100a kernels and the shards are concatenated; the result must
  match the oracle on the whole batch.
* On two or more GPUs: ``torchrun`` with two NCCL ranks, each holding only its
  own heads' pages, gathers the outputs; both ranks check the full result.
"""

import os
import subprocess
import tempfile
import sys
import textwrap

import numpy as np
import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200.sharded import ShardedPagedAttention, shard_cache, shard_queries
from decodekernels_b200.testing import make_paged_kv
from gpu_helpers import assert_attention_close, oracle_dense

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("layout", ["vllm", "hnd", "nhd"])
def test_emulated_ranks_on_one_gpu(world, layout):
    seq_lens = [1, 513, 3000, 0, 1200]
    kv = make_paged_kv(seq_lens, 8, 128, 16, torch.float16, "cuda", layout=layout, seed=world)
    g = torch.Generator(device="cuda").manual_seed(world)
    q = torch.randn(len(seq_lens), 64, 128, generator=g, device="cuda", dtype=torch.float16)
    parts = []
    for r in range(world):
        attn = ShardedPagedAttention(64, 8, rank=r, world=world)
        s = attn.shard
        parts.append(attn(shard_queries(q, s), shard_cache(kv.k_cache, s), shard_cache(kv.v_cache, s),
                          kv.block_tables, kv.seq_lens))
    out = torch.cat(parts, dim=1)
    assert_attention_close(out, oracle_dense(q, kv), torch.float16, f"{world} shards, {layout}")


_SCRIPT = textwrap.dedent(
    """
    import datetime, os, sys
    sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
    import numpy as np, torch, torch.distributed as dist
    from decodekernels_b200.sharded import ShardedPagedAttention
    from decodekernels_b200.testing import make_paged_kv
    from gpu_helpers import assert_attention_close, oracle_dense
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    lens = [7, 900, 4000, 64]
    full = make_paged_kv(lens, 8, 128, 16, torch.bfloat16, "cpu", layout="vllm", seed=11)
    q = torch.randn(len(lens), 64, 128, generator=torch.Generator().manual_seed(12), dtype=torch.bfloat16)
    attn = ShardedPagedAttention(64, 8)
    s = attn.shard
    # this rank allocates only its own heads' pages (vLLM layout: [blocks, heads, bs, 2D])
    buf = torch.cat([full.k_cache, full.v_cache], dim=-1).transpose(1, 2)[:, s.kv_slice].contiguous().cuda()
    k, v = buf.transpose(1, 2).split(128, dim=-1)
    out = attn(q[:, s.q_slice].cuda(), k, v, full.block_tables.cuda(), full.seq_lens.cuda(), gather=True)
    torch.cuda.synchronize()
    ref = oracle_dense(q, full)
    assert_attention_close(out, ref, torch.bfloat16, "rank %d gathered" % rank)
    dist.barrier()
    dist.destroy_process_group()
    print("rank", rank, "ok")
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_gather():
    script = _SCRIPT.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    path = tempfile.gettempdir()
    f = os.path.join(path, "sharded_nccl_case.py")
    with open(f, "w") as fh:
        fh.write(script)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533", f],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok") == 2


def test_peer_gather_world_one_copies_local_heads():
    """dk_gather_heads with a group of one: the local heads land in out
    (through the receive slot), call after call, with any out strides."""
    from decodekernels_b200 import capi

    n, hq, d = 5, 16, 128
    state = torch.zeros(4, dtype=torch.int32, device="cuda")
    buf = torch.zeros(256 + 2 * n * hq * d * 2, dtype=torch.uint8, device="cuda")
    for it in range(3):
        local = torch.randn(n, hq, d, device="cuda").to(torch.bfloat16)
        wide = torch.full((n, hq + 3, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        out = wide[:, 1:hq + 1]  # strided destination
        capi.gather_heads(local, [buf.data_ptr() + 256], [buf.data_ptr()], state, out, rank=0, world=1)
        torch.cuda.synchronize()
        assert torch.equal(out, local)
        assert int(state[0].item()) == it + 1 and int(state[3].item()) == 0


@pytest.mark.parametrize("counters", [False, True])
def test_fused_decode_gather_world_one_equals_decode(counters):
    """dk_paged_attention_decode_gather with a group of one: the decode's
    output stores go to the receive slot, the small kernel copies them to out;
    bit-identical to the plain decode, call after call (both slot parities),
    with the merge kernel or the single-launch merge, and with no sequences."""
    from decodekernels_b200 import capi

    lens = [1, 513, 3000, 0, 1200, 64]
    kv = make_paged_kv(lens, 2, 128, 16, torch.bfloat16, "cuda", layout="vllm", seed=3)
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(len(lens), 16, 128, generator=g, device="cuda").to(torch.bfloat16)
    n, hq, d = q.shape
    ws = dk.alloc_workspace(n, hq, d, 3000, "cuda", num_kv_heads=2, block_size=16, merge_counters=counters)
    want = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=3000,
                                     workspace=ws)
    state = torch.zeros(4, dtype=torch.int32, device="cuda")
    buf = torch.zeros(256 + 2 * n * hq * d * 2, dtype=torch.uint8, device="cuda")
    for it in range(3):
        wide = torch.full((n, hq + 2, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        out = wide[:, 2:]
        capi.decode_gather(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, d**-0.5, 3000, ws,
                           [buf.data_ptr() + 256], [buf.data_ptr()], state, out, rank=0, world=1)
        torch.cuda.synchronize()
        assert torch.equal(out, want), f"call {it}"
        assert int(state[0].item()) == it + 1 and int(state[3].item()) == 0
    empty = torch.empty(0, hq, d, dtype=torch.bfloat16, device="cuda")
    capi.decode_gather(q[:0], kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, d**-0.5, 3000, ws,
                       [buf.data_ptr() + 256], [buf.data_ptr()], state, empty, rank=0, world=1)
    torch.cuda.synchronize()
    assert int(state[0].item()) == 4  # the collective still ran


def test_peer_gather_wait_gives_up_and_reports():
    """One GPU, world 2: the second rank's flag is a word nothing sets, so the
    gather's bounded wait runs out, records the give-up in state[3] and
    returns; this rank's heads are in place and the context stays usable."""
    from decodekernels_b200 import capi

    n, hpr, d = 3, 4, 64
    slot = n * 2 * hpr * d * 2
    mine = torch.zeros(256 + 2 * slot, dtype=torch.uint8, device="cuda")
    other = torch.zeros_like(mine)  # stands in for a peer that never calls
    state = torch.zeros(4, dtype=torch.int32, device="cuda")
    local = torch.randn(n, hpr, d, device="cuda").to(torch.float16)
    out = torch.zeros(n, 2 * hpr, d, dtype=torch.float16, device="cuda")
    capi.gather_heads(local, [mine.data_ptr() + 256, other.data_ptr() + 256], [mine.data_ptr(), other.data_ptr()],
                      state, out, rank=0, world=2, wait_limit_ms=100)
    torch.cuda.synchronize()
    assert int(state[3].item()) >= 1  # gave up instead of hanging
    assert torch.equal(out[:, :hpr], local)
    other_flags = other[:8].view(torch.int32)
    assert int(other_flags[0].item()) == 1 and int(other_flags[1].item()) == 0  # we signalled; the peer never did
    kv = make_paged_kv([100], 1, 128, 16, torch.bfloat16, "cuda")
    q = torch.randn(1, 8, 128, device="cuda").to(torch.bfloat16)
    assert_attention_close(dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens),
                           oracle_dense(q, kv), torch.bfloat16, "after a given-up gather")


_P2P_GATHER_SCRIPT = textwrap.dedent(
    """
    import datetime, os, sys
    sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
    import torch, torch.distributed as dist
    from decodekernels_b200.sharded import ShardedPagedAttention, shard_cache, shard_queries
    from decodekernels_b200.testing import make_paged_kv
    from gpu_helpers import assert_attention_close, oracle_dense
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    L = 3000
    lens0 = [7, 900, L, 64, 0, 1500, 513]
    full = make_paged_kv([L] * len(lens0), 8, 128, 16, torch.float16, "cpu", layout="vllm", seed=41)
    q_cpu = torch.randn(len(lens0), 32, 128, generator=torch.Generator().manual_seed(42), dtype=torch.float16)
    p2p = ShardedPagedAttention(32, 8, exchange="p2p")
    nccl = ShardedPagedAttention(32, 8)
    s = p2p.shard
    k, v = shard_cache(full.k_cache, s).cuda(), shard_cache(full.v_cache, s).cuda()  # this rank's heads only
    q = shard_queries(q_cpu, s).contiguous().cuda()
    bt = full.block_tables.cuda()
    lens = torch.tensor(lens0, dtype=torch.int32, device="cuda")
    out = torch.empty(len(lens0), 32, 128, dtype=torch.float16, device="cuda")
    # one workspace kind for every path (merge counters: the single-launch
    # merge), so their plans match and the outputs can be compared bit for bit
    import decodekernels_b200 as dk
    ws = dk.alloc_workspace(len(lens0), 16, 128, L, "cuda", num_kv_heads=4, block_size=16, merge_counters=True)

    def step():
        p2p(q, k, v, bt, lens, max_seq_len=L, workspace=ws, gather=True, gathered_out=out)

    g = torch.Generator().manual_seed(43)
    for it in range(4):  # eager calls: the device-side call counter advances in lockstep
        lens.copy_(torch.randint(0, L + 1, (len(lens0),), generator=g, dtype=torch.int32))
        step()
        torch.cuda.synchronize()
        full.seq_lens.copy_(lens.cpu())
        assert_attention_close(out, oracle_dense(q_cpu, full), torch.float16, "rank %d eager %d" % (rank, it))
        ref = nccl(q, k, v, bt, lens, max_seq_len=L, workspace=ws, gather=True)
        assert torch.equal(ref, out), "fused p2p and NCCL gathers differ"
        local = nccl(q, k, v, bt, lens, max_seq_len=L, workspace=ws)
        assert torch.equal(p2p.gather(local), out), "fused and unfused p2p gathers differ"
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        step()
    torch.cuda.current_stream().wait_stream(st)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for it in range(3):
        lens.copy_(torch.randint(0, L + 1, (len(lens0),), generator=g, dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        full.seq_lens.copy_(lens.cpu())
        assert_attention_close(out, oracle_dense(q_cpu, full), torch.float16, "rank %d graph %d" % (rank, it))
    del graph
    assert p2p.p2p_errors() == 0
    dist.barrier()
    dist.destroy_process_group()
    print("rank", rank, "ok")
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_peer_memory_gather():
    """Two GPUs: the gather fused into the decode's output stores equals the
    separate peer-memory gather and NCCL's, and the oracle, eagerly and under
    CUDA-graph replay."""
    script = _P2P_GATHER_SCRIPT.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    path = tempfile.gettempdir()
    f = os.path.join(path, "head_sharded_p2p_case.py")
    with open(f, "w") as fh:
        fh.write(script)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29541", f],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok") == 2
