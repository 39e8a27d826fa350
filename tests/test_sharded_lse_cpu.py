"""CPU: sequence (block-striped) sharding -- the oracle's LSE partials and
merge, the product's striping helper, and the gather-and-merge logic of
SequenceShardedPagedAttention on world-size-2 ``gloo`` ranks (the CPU oracle
stands in for the CUDA kernels, since this file tests the distribution
logic only).  A rank that dies before the exchange makes the other fail
within the process-group timeout instead of hanging."""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from decodekernels_b200.sharded import SequenceShardedPagedAttention, stripe_tables
from decodekernels_b200.testing import make_paged_kv, make_queries
from oracle import oracle
from oracle import sharded_lse as sl


def _problem(seed=3):
    kv = make_paged_kv([5, 70, 300, 0, 16, 17, 1000], 2, 64, 16, torch.float32, "cpu", layout="nhd", seed=seed)
    q = make_queries(7, 8, 64, torch.float32, seed=seed + 1)
    return q, kv


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_striped_partials_merge_to_dense(world):
    q, kv = _problem()
    want = oracle.paged_attention_dense(q, kv.k_cache, kv.v_cache, kv.block_tables.numpy(), kv.seq_lens.numpy())
    o_parts, lse_parts = [], []
    total = np.zeros(7, dtype=np.int64)
    for r in range(world):
        bt, lens = sl.stripe(kv.block_tables.numpy(), kv.seq_lens.numpy(), 16, r, world)
        total += lens
        o, lse = sl.attention_lse(q, kv.k_cache, kv.v_cache, bt, lens)
        o_parts.append(o)
        lse_parts.append(lse)
    assert np.array_equal(total, kv.seq_lens.numpy())
    o, lse = sl.merge_lse(o_parts, lse_parts)
    np.testing.assert_allclose(o, want, atol=2e-6, rtol=1e-5)
    o_all, lse_all = sl.attention_lse(q, kv.k_cache, kv.v_cache, kv.block_tables.numpy(), kv.seq_lens.numpy())
    np.testing.assert_allclose(lse[np.isfinite(lse_all)], lse_all[np.isfinite(lse_all)], rtol=1e-5)
    assert np.all(np.isneginf(lse[3])) and not o[3].any()


@pytest.mark.parametrize("world", [2, 3, 8])
def test_product_striping_matches_oracle(world):
    q, kv = _problem()
    for r in range(world):
        bt, lens = stripe_tables(kv.block_tables, kv.seq_lens, 16, r, world)
        want_bt, want_lens = sl.stripe(kv.block_tables.numpy(), kv.seq_lens.numpy(), 16, r, world)
        assert bt.is_contiguous() and bt.dtype == torch.int32 and lens.dtype == torch.int32
        assert np.array_equal(bt.numpy(), want_bt) and np.array_equal(lens.numpy(), want_lens)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lse_fn(q, k, v, bt, lens, scale=None, max_seq_len=None, partial=None, workspace=None):
    o, lse = sl.attention_lse(q, k, v, bt.numpy(), lens.numpy(), scale=scale)
    out = torch.zeros(q.shape[0], q.shape[1], q.shape[2] + 4)
    out[..., : q.shape[2]] = torch.from_numpy(o)
    out[..., q.shape[2]] = torch.from_numpy(lse)
    return out


def _merge_fn(parts, out=None, dtype=torch.float32):
    D = parts.shape[-1] - 4
    o, _ = sl.merge_lse(parts[..., :D].numpy(), parts[..., D].numpy())
    return torch.from_numpy(o)


def _worker(rank, world, port, outdir, mode):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    q, kv = _problem()
    attn = SequenceShardedPagedAttention(block_size=16, lse_fn=_lse_fn, merge_fn=_merge_fn)
    bt, lens = stripe_tables(kv.block_tables, kv.seq_lens, 16, attn.rank, attn.world)
    if mode == "dead" and rank == 1:
        os._exit(0)  # leaves without joining the exchange
    try:
        out = attn(q, kv.k_cache, kv.v_cache, bt, lens, scale=64**-0.5, max_seq_len=1000)
        torch.save(out, os.path.join(outdir, f"rank{rank}.pt"))
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


def test_two_gloo_ranks_match_the_whole_batch():
    outdir = _run("ok")
    q, kv = _problem()
    want = oracle.paged_attention_dense(q, kv.k_cache, kv.v_cache, kv.block_tables.numpy(), kv.seq_lens.numpy())
    for r in range(2):
        got = torch.load(os.path.join(outdir, f"rank{r}.pt"))
        np.testing.assert_allclose(got.numpy(), want, atol=2e-6, rtol=1e-5)


def test_dead_rank_fails_the_exchange_instead_of_hanging():
    outdir = _run("dead")
    assert os.path.exists(os.path.join(outdir, "rank0.err")), "rank 0 finished an exchange whose peer had exited"


@pytest.mark.parametrize("world", [1, 2, 3])
def test_striped_workload_builder(world):
    """bench.py's sequence-sharded batches: the ranks' lengths add up to the
    config's, every rank holds the same queries, and each table only names
    blocks of the rank's own pool."""
    from decodekernels_b200 import workloads

    full = workloads.seq_lens("c1")
    total = np.zeros(len(full), dtype=np.int64)
    q0 = None
    for r in range(world):
        b = workloads.make_striped("c1", "cpu", stripe=(r, world))
        total += np.array(b.lens)
        assert b.kv.seq_lens.tolist() == b.lens
        assert int(b.kv.block_tables.max()) < b.kv.k_cache.shape[0]
        q0 = b.q if q0 is None else q0
        assert torch.equal(b.q, q0)
        want_bt, want_lens = sl.stripe(np.zeros((len(full), 64), np.int32), full, 16, r, world)
        assert b.lens == want_lens.tolist()
    assert total.tolist() == full
