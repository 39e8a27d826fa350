"""GPU: sequence-sharded decode with the real kernels.

* ``dk.paged_attention_decode_lse`` against the oracle's (o, lse) on every
  path (single pass, split with the merge kernel, single-launch merge, the
  CUDA-core path), head sizes and layouts, empty sequences included.
* ``dk.merge_lse`` against the oracle's log-sum-exp merge.
* Block-striped shards emulated on one GPU (world 2, 4, 8, including MQA with
  one KV head): the merged output matches the oracle on whole sequences.
* Two NCCL ranks (when two GPUs are visible), each holding only its own
  blocks, exchange partials and both reproduce the whole batch.
"""

import ctypes
import os
import subprocess
import tempfile
import sys
import textwrap

import numpy as np
import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import capi
from decodekernels_b200.sharded import SequenceShardedPagedAttention, stripe_tables
from decodekernels_b200.testing import make_paged_kv
from gpu_helpers import alloc_ws, assert_attention_close, oracle_dense
from oracle import sharded_lse as sl

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _q(n, hq, d, dtype, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(n, hq, d, generator=g, device="cuda", dtype=dtype)


def _check_partial(partial, q, kv, what, scale=None):
    D = q.shape[-1]
    o_want, lse_want = sl.attention_lse(q.cpu(), kv.k_cache.cpu(), kv.v_cache.cpu(), kv.block_tables.cpu().numpy(),
                                        kv.seq_lens.cpu().numpy(), scale=scale)
    got = partial.cpu().numpy()
    o, lse = got[..., :D], got[..., D]
    err = np.abs(o - o_want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, f"{what}: o max {err.max():.2e} mean {err.mean():.2e}"
    empty = np.isneginf(lse_want)
    assert np.array_equal(np.isneginf(lse), empty), f"{what}: -inf lse where the sequence is (not) empty"
    assert not o[empty].any()
    np.testing.assert_allclose(lse[~empty], lse_want[~empty], atol=2e-3, rtol=1e-4, err_msg=what)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim,group,layout", [(128, 8, "vllm"), (64, 1, "nhd"), (256, 8, "hnd")])
@pytest.mark.parametrize("path", ["single", "planner", "ps64", "fused", "simt"])
def test_decode_lse_matches_oracle(dtype, head_dim, group, layout, path):
    lens = [1, 0, 63, 64, 65, 700, 2500, 17]
    kv = make_paged_kv(lens, 2, head_dim, 16, dtype, "cuda", layout=layout, seed=head_dim)
    q = _q(len(lens), 2 * group, head_dim, dtype, seed=group)
    n, hq, d = q.shape
    partial = torch.full((n, hq, d + 4), float("nan"), dtype=torch.float32, device="cuda")
    L = max(lens)
    ps, flags, simt = 0, 0, False
    if path == "single":
        ws = None
    elif path == "ps64":
        ps = 64
        ws = alloc_ws(n, hq, d, -(-L // 64), q.device)
    else:
        ws = alloc_ws(n, hq, d, capi.num_partitions(n, 2, d, 16, L), q.device)
        if path == "fused":
            ws = (*ws, torch.zeros(n * 2, dtype=torch.int32, device="cuda"))
            flags = capi.DK_FLAG_FORCE_FUSED_MERGE
        simt = path == "simt"
    a = capi.make_args(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, d**-0.5, L, partial, ws, ps, simt,
                       flags)
    rc = capi.load().dk_paged_attention_decode_lse(ctypes.byref(a), partial.data_ptr(),
                                                   torch.cuda.current_stream().cuda_stream)
    assert rc == 0, capi.last_error()
    torch.cuda.synchronize()
    _check_partial(partial, q, kv, f"{path} D{head_dim} {layout}")
    if path == "fused":
        assert int(ws[3].abs().sum().item()) == 0


def test_decode_lse_torch_op():
    kv = make_paged_kv([0, 3000, 40], 4, 128, 32, torch.bfloat16, "cuda", layout="vllm")
    q = _q(3, 16, 128, torch.bfloat16)
    partial = dk.paged_attention_decode_lse(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    torch.cuda.synchronize()
    assert partial.shape == (3, 16, 132) and partial.dtype == torch.float32
    _check_partial(partial, q, kv, "torch op")


@pytest.mark.parametrize("R", [1, 2, 5, 8])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_merge_lse_matches_oracle(R, D):
    g = torch.Generator(device="cuda").manual_seed(R * D)
    n, hq = 5, 6
    parts = torch.randn(R, n, hq, D + 4, generator=g, device="cuda")
    parts[..., D] = torch.randn(R, n, hq, generator=g, device="cuda") * 20
    parts[0, 1, :, D] = -float("inf")  # an empty shard
    parts[:, 2, 3, D] = -float("inf")  # empty everywhere
    parts[:, 2, 3, :D] = 0.0
    parts[0, 1, :, :D] = 0.0
    o_want, lse_want = sl.merge_lse(parts[..., :D].cpu().numpy(), parts[..., D].cpu().numpy())
    for dtype in (torch.float16, torch.bfloat16):
        out = dk.merge_lse(parts, dtype=dtype)
        torch.cuda.synchronize()
        assert_attention_close(out, o_want, dtype, f"merge R={R} {dtype}")
    merged = torch.empty(n, hq, D + 4, device="cuda")
    dk.merge_lse(parts, out=merged)
    torch.cuda.synchronize()
    got = merged.cpu().numpy()
    np.testing.assert_allclose(got[..., :D], o_want, atol=1e-5, rtol=1e-5)
    fin = np.isfinite(lse_want)
    np.testing.assert_allclose(got[..., D][fin], lse_want[fin], atol=1e-4, rtol=1e-5)
    assert np.isneginf(got[2, 3, D]) and not got[2, 3, :D].any()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("hkv,hq,layout", [(8, 64, "vllm"), (1, 8, "nhd")])
def test_emulated_striped_ranks_on_one_gpu(world, hkv, hq, layout):
    lens = [1, 513, 3000, 0, 1200, 16, 17]
    kv = make_paged_kv(lens, hkv, 128, 16, torch.bfloat16, "cuda", layout=layout, seed=world)
    q = _q(len(lens), hq, 128, torch.bfloat16, seed=world)
    parts = []
    for r in range(world):
        attn = SequenceShardedPagedAttention(block_size=16, rank=r, world=world)
        bt, lens_r = stripe_tables(kv.block_tables, kv.seq_lens, 16, r, world)
        parts.append(attn.partial(q, kv.k_cache, kv.v_cache, bt, lens_r, max_seq_len=max(lens)))
    out = dk.merge_lse(torch.stack(parts), dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert_attention_close(out, oracle_dense(q, kv), torch.bfloat16, f"{world} striped shards")
    full = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    assert (out.float() - full.float()).abs().max().item() <= 2e-2


_SCRIPT = textwrap.dedent(
    """
    import datetime, os, sys
    sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
    import torch, torch.distributed as dist
    from decodekernels_b200.sharded import SequenceShardedPagedAttention, stripe_tables
    from decodekernels_b200.testing import make_paged_kv
    from gpu_helpers import assert_attention_close, oracle_dense
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    lens = [7, 900, 4000, 64, 0]
    full = make_paged_kv(lens, 1, 256, 32, torch.bfloat16, "cpu", layout="nhd", seed=21)  # MQA: one KV head
    q = torch.randn(len(lens), 8, 256, generator=torch.Generator().manual_seed(22), dtype=torch.bfloat16)
    attn = SequenceShardedPagedAttention(block_size=32)
    bt, lens_r = stripe_tables(full.block_tables, full.seq_lens, 32, attn.rank, attn.world)
    # this rank allocates only its own blocks: compact them and renumber its table
    used = sorted(set(int(b) for b in bt.flatten().tolist()))
    remap = torch.full((full.k_cache.shape[0],), 0, dtype=torch.int32)
    remap[torch.tensor(used, dtype=torch.long)] = torch.arange(len(used), dtype=torch.int32)
    k = full.k_cache[used].cuda()
    v = full.v_cache[used].cuda()
    out = attn(q.cuda(), k, v, remap[bt.long()].cuda(), lens_r.cuda(), max_seq_len=max(lens))
    torch.cuda.synchronize()
    assert_attention_close(out, oracle_dense(q, full), torch.bfloat16, "rank %d" % rank)
    dist.barrier()
    dist.destroy_process_group()
    print("rank", rank, "ok")
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_exchange_partials():
    script = _SCRIPT.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    path = tempfile.gettempdir()
    f = os.path.join(path, "seq_sharded_nccl_case.py")
    with open(f, "w") as fh:
        fh.write(script)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29537", f],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok") == 2


def test_peer_exchange_wait_gives_up_and_reports():
    """One GPU, world 2: the second rank's flag is a word nothing sets, so the
    exchange's bounded wait runs out, records the give-up in state[3] and
    returns; the context stays usable."""
    n, hq, d = 3, 8, 128
    partial = torch.zeros(n, hq, d + 4, device="cuda")
    partial[..., d] = 0.0
    block = n * hq * (d + 4)
    mine = torch.zeros(64 + 2 * 2 * block, device="cuda")
    other = torch.zeros_like(mine)  # stands in for a peer that never calls
    recv = [mine.data_ptr() + 256, other.data_ptr() + 256]
    flags = [mine.data_ptr(), other.data_ptr()]
    state = torch.zeros(4, dtype=torch.int32, device="cuda")
    out = torch.empty(n, hq, d, dtype=torch.bfloat16, device="cuda")
    capi.exchange_merge_lse(partial, recv, flags, state, out, rank=0, world=2, wait_limit_ms=100)
    torch.cuda.synchronize()
    assert int(state[3].item()) >= 1  # gave up instead of hanging
    other_flags = other.view(torch.int32)
    assert int(other_flags[0].item()) == 1 and int(other_flags[1].item()) == 0  # we signalled; the peer never did
    kv = make_paged_kv([100], 1, 128, 16, torch.bfloat16, "cuda")
    q = _q(1, 8, 128, torch.bfloat16)
    assert_attention_close(dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens),
                           oracle_dense(q, kv), torch.bfloat16, "after a given-up exchange")


_P2P_SCRIPT = textwrap.dedent(
    """
    import datetime, os, sys
    sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
    import torch, torch.distributed as dist
    from decodekernels_b200.sharded import SequenceShardedPagedAttention, stripe_tables
    from decodekernels_b200.testing import make_paged_kv
    from gpu_helpers import assert_attention_close, oracle_dense
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    L = 4000
    lens0 = [7, 900, L, 64, 0, 1500]
    full = make_paged_kv([L] * len(lens0), 2, 128, 16, torch.bfloat16, "cpu", layout="nhd", seed=31)
    q_cpu = torch.randn(len(lens0), 16, 128, generator=torch.Generator().manual_seed(32), dtype=torch.bfloat16)
    q = q_cpu.cuda()
    attn = SequenceShardedPagedAttention(block_size=16, exchange="p2p")
    nccl = SequenceShardedPagedAttention(block_size=16)
    k, v = full.k_cache.cuda(), full.v_cache.cuda()  # whole cache here; each rank reads only its blocks
    bt_full = full.block_tables.cuda()
    lens = torch.tensor(lens0, dtype=torch.int32, device="cuda")
    out = torch.empty(len(lens0), 16, 128, dtype=torch.bfloat16, device="cuda")

    def step():
        bt, ll = stripe_tables(bt_full, lens, 16, attn.rank, attn.world)
        attn(q, k, v, bt, ll, max_seq_len=L, out=out)

    g = torch.Generator().manual_seed(33)
    for it in range(4):  # eager calls: the device-side call counter advances in lockstep
        lens.copy_(torch.randint(0, L + 1, (len(lens0),), generator=g, dtype=torch.int32))
        step()
        torch.cuda.synchronize()
        full.seq_lens.copy_(lens.cpu())
        assert_attention_close(out, oracle_dense(q_cpu, full), torch.bfloat16, "rank %d eager %d" % (rank, it))
        bt, ll = stripe_tables(bt_full, lens, 16, nccl.rank, nccl.world)
        ref = nccl(q, k, v, bt, ll, max_seq_len=L)
        assert (ref.float() - out.float()).abs().max().item() <= 1e-2
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for it in range(3):
        lens.copy_(torch.randint(0, L + 1, (len(lens0),), generator=g, dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        full.seq_lens.copy_(lens.cpu())
        assert_attention_close(out, oracle_dense(q_cpu, full), torch.bfloat16, "rank %d graph %d" % (rank, it))
    del graph
    assert attn.p2p_errors() == 0
    dist.barrier()
    dist.destroy_process_group()
    print("rank", rank, "ok")
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_peer_memory_exchange():
    script = _P2P_SCRIPT.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    path = tempfile.gettempdir()
    f = os.path.join(path, "seq_sharded_p2p_case.py")
    with open(f, "w") as fh:
        fh.write(script)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29539", f],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok") == 2
