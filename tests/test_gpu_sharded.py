"""GPU: KV-head sharding with the real kernels.

* On one GPU: every rank's shard (strided views of one cache) is computed
  with the sm_100a kernels and the shards are concatenated; the result must
  match the oracle on the whole batch.
* On two or more GPUs: ``torchrun`` with two NCCL ranks, each holding only its
  own heads' pages, gathers the outputs; both ranks check the full result.
"""

import os
import subprocess
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
    path = os.path.join(ROOT, "gpurun_out") if os.path.isdir(os.path.join(ROOT, "gpurun_out")) else "/tmp"
    f = os.path.join(path, "sharded_nccl_case.py")
    with open(f, "w") as fh:
        fh.write(script)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533", f],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok") == 2
