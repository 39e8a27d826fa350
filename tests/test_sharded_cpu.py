"""CPU: the KV-head sharding layer with world-size-2 ``gloo`` ranks.

Each rank computes its own heads (the CPU oracle stands in for the CUDA
kernel here, since this file tests only the distribution logic) and the
all-gather reassembles the full output, which must equal the oracle on the
whole batch.  A rank that dies before the collective must make the other
rank fail within the process-group timeout instead of hanging.
"""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from decodekernels_b200.sharded import ShardedPagedAttention, head_shard, shard_cache, shard_queries


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_fn(q, k, v, bt, sl, scale=None, max_seq_len=None, out=None, workspace=None):
    from oracle import oracle

    return torch.from_numpy(oracle.paged_attention_dense(q, k, v, bt.numpy(), sl.numpy(), scale=scale))


def _problem():
    from decodekernels_b200.testing import make_paged_kv, make_queries

    kv = make_paged_kv([5, 70, 300, 0], 4, 64, 16, torch.float32, "cpu", layout="vllm", seed=3)
    q = make_queries(4, 16, 64, torch.float32, seed=4)
    return q, kv


def _worker(rank, world, port, outdir, mode):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    q, kv = _problem()
    attn = ShardedPagedAttention(16, 4, attention_fn=_oracle_fn)
    s = attn.shard
    q_l, k_l, v_l = shard_queries(q, s), shard_cache(kv.k_cache, s), shard_cache(kv.v_cache, s)
    if mode == "dead" and rank == 1:
        os._exit(0)  # leaves without joining the collective
    try:
        local = attn(q_l, k_l, v_l, kv.block_tables, kv.seq_lens, scale=64**-0.5)
        full = attn(q_l, k_l, v_l, kv.block_tables, kv.seq_lens, scale=64**-0.5, gather=True)
        torch.save({"local": local, "full": full}, os.path.join(outdir, f"rank{rank}.pt"))
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(outdir, f"rank{rank}.err"), "w") as f:
            f.write(repr(e))
    if mode != "dead":
        dist.destroy_process_group()


def _run(mode):
    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, outdir, mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank hung")
    return outdir


def test_shard_math():
    s = head_shard(64, 8, 3, 4)
    assert (s.kv_slice, s.q_slice) == (slice(6, 8), slice(48, 64))
    assert head_shard(32, 8, 0, 1).kv_per_rank == 8
    with pytest.raises(ValueError):
        head_shard(8, 1, 0, 2)  # MQA cannot be head-sharded
    with pytest.raises(ValueError):
        head_shard(64, 8, 4, 4)


def test_two_gloo_ranks_match_the_whole_batch():
    outdir = _run("ok")
    q, kv = _problem()
    want = _oracle_fn(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale=64**-0.5)
    for r in range(2):
        got = torch.load(os.path.join(outdir, f"rank{r}.pt"))
        np.testing.assert_allclose(got["full"].numpy(), want.numpy(), atol=1e-6, rtol=1e-6)
        np.testing.assert_allclose(got["local"].numpy(), want[:, r * 8:(r + 1) * 8].numpy(), atol=1e-6, rtol=1e-6)


def test_dead_rank_fails_the_collective_instead_of_hanging():
    outdir = _run("dead")
    err = os.path.join(outdir, "rank0.err")
    assert os.path.exists(err), "rank 0 finished a gather whose peer had exited"


def test_head_sharded_exchange_must_be_known():
    from decodekernels_b200.sharded import ShardedPagedAttention

    with pytest.raises(ValueError, match="exchange"):
        ShardedPagedAttention(32, 8, rank=0, world=1, exchange="mpi")
    attn = ShardedPagedAttention(32, 8, rank=0, world=1, exchange="p2p")
    local = torch.randn(3, 32, 64)
    assert attn.gather(local) is local  # a group of one needs no exchange
    dst = torch.empty_like(local)
    assert attn.gather(local, dst) is dst and torch.equal(dst, local)
