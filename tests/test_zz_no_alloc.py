"""GPU: the decode entry point for callers that cannot allocate device memory.

Some callers of this library may not allocate: inference runtimes and plugin
hosts that give a kernel only its inputs and outputs and own every other byte
of device memory, and host languages whose FFI has no CUDA allocator.
``dk_paged_attention_decode_noalloc`` serves them: it takes no workspace and
keeps the split-K partials in the library's static scratch array.

These tests call it through the C ABI and compare it with the regular entry
point (which gets a workspace allocated here), on two calls in a row with
different batches, so the second call starts from the first call's leftover
scratch.  Small calls also use the library's own merge counters; the compact
grid cases (an e4m3 cache, and DK_FLAG_PERSISTENT) run the same call three
times and require identical results, which holds only if the counters are
zero whenever a call starts.  The file is named to run last; it passes alone
and after the rest.
"""

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


def _batch(seq_lens, seed, dtype, layout):
    kv = make_paged_kv(seq_lens, 8, 128, 16, dtype, "cuda", layout=layout, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 100)
    q = torch.randn(len(seq_lens), 32, 128, generator=g, device="cuda", dtype=dtype)
    return q, kv


def _regular(q, kv, max_len, k=None, v=None, flags=0, scales=(1.0, 1.0)):
    n, hq, d = q.shape
    k = kv.k_cache if k is None else k
    v = kv.v_cache if v is None else v
    parts = capi.num_partitions(n, k.shape[2], d, kv.block_size, max_len)
    out = torch.full_like(q, float("nan"))
    capi.decode(q, k, v, kv.block_tables, kv.seq_lens, d**-0.5, max_len, out, alloc_ws(n, hq, d, parts, q.device),
                flags=flags, k_scale=scales[0], v_scale=scales[1])
    return out


def test_noalloc_matches_regular_entry_point_on_two_calls_in_a_row():
    batches = [
        _batch([1, 511, 512, 513, 0, 3000, 4096, 77], seed=1, dtype=torch.bfloat16, layout="nhd"),
        _batch([2048, 5, 0, 1500, 4000, 1024], seed=2, dtype=torch.float16, layout="vllm"),
    ]
    for q, kv in batches:
        max_len = int(kv.seq_lens.max())
        plan = capi.plan(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, 128**-0.5, max_len,
                         torch.empty_like(q), alloc_ws(q.shape[0], q.shape[1], 128, 64, q.device))
        assert plan["split"] == 1  # the scratch is really used
        want = _regular(q, kv, max_len)
        got = torch.full_like(q, float("nan"))
        capi.decode_noalloc(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, 128**-0.5, max_len, got)
        torch.cuda.synchronize()
        assert_attention_close(got, want.float().cpu().numpy(), q.dtype, "no-alloc vs regular")
        assert_attention_close(got, oracle_dense(q, kv), q.dtype, "no-alloc vs oracle")
    assert capi.wait_timeouts(0) == 0


def test_noalloc_rejects_calls_beyond_its_scratch():
    # 256 sequences x 64 query heads x 64 partitions of 512 tokens need ~545 MB of
    # partials, more than the static scratch.  All lengths are 0, so even a launch
    # would read no cache; the call must be refused before launching anything.
    n, hq, d, L = 256, 64, 128, 32768
    q = torch.zeros(n, hq, d, dtype=torch.float16, device="cuda")
    out = torch.full_like(q, 7.0)
    k = torch.zeros(1, 16, 8, d, dtype=torch.float16, device="cuda")
    tables = torch.zeros(n, L // 16, dtype=torch.int32, device="cuda")
    lens = torch.zeros(n, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="static scratch holds"):
        capi.decode_noalloc(q, k, k, tables, lens, d**-0.5, L, out)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing ran


def test_noalloc_refuses_a_workspace():
    q, kv = _batch([10, 20], seed=3, dtype=torch.bfloat16, layout="nhd")
    args = capi.make_args(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, 0.1, 20, torch.empty_like(q),
                          alloc_ws(2, 32, 128, 2, q.device))
    import ctypes

    rc = capi.load().dk_paged_attention_decode_noalloc(ctypes.byref(args), None)
    assert rc == 1 and "takes no workspace" in capi.last_error()


KS, VS = 0.02, 0.015


@pytest.mark.parametrize("case", ["e4m3_compact", "persistent"])
def test_noalloc_compact_grid_with_library_counters(case):
    # Few (sequence, KV head) pairs and long sequences: 16 partitions of 1024
    # tokens, a merge small enough for the single-launch merge, so the call
    # uses the library-owned merge counters.  e4m3 caches take the compact grid
    # by default there; DK_FLAG_PERSISTENT takes it (one wave, several items
    # per CTA) for a 16-bit cache.  The same call runs twice more: equal
    # results show the counters were zero at the start of every call.
    lens = [16384, 9000, 0, 1, 12000, 3000, 16000, 777]
    q, kv = _batch(lens, seed=5, dtype=torch.float16, layout="vllm")
    max_len = max(lens)
    if case == "e4m3_compact":
        k, v = fp8_caches(kv, "vllm", KS, VS)
        flags, scales = 0, (KS, VS)
        want = oracle_dense_fp8(q, kv, k, v, KS, VS)
    else:
        k, v = kv.k_cache, kv.v_cache
        flags, scales = capi.DK_FLAG_PERSISTENT, (1.0, 1.0)
        want = oracle_dense(q, kv)
    counters = torch.zeros(len(lens) * 8, dtype=torch.int32, device="cuda")
    parts = capi.num_partitions(len(lens), 8, 128, 16, max_len)
    plan = capi.plan(q, k, v, kv.block_tables, kv.seq_lens, 128**-0.5, max_len, torch.empty_like(q),
                     (*alloc_ws(len(lens), 32, 128, parts, q.device), counters), flags=flags, k_scale=scales[0],
                     v_scale=scales[1])
    assert plan["split"] == 1 and plan["launches"] == 1 and plan["num_partitions"] >= 16, plan
    regular = _regular(q, kv, max_len, k, v, flags, scales)
    runs = []
    for _ in range(3):
        got = torch.full_like(q, float("nan"))
        capi.decode_noalloc(q, k, v, kv.block_tables, kv.seq_lens, 128**-0.5, max_len, got, flags=flags,
                            k_scale=scales[0], v_scale=scales[1])
        torch.cuda.synchronize()
        runs.append(got)
    assert torch.equal(runs[0], runs[1]) and torch.equal(runs[1], runs[2]), "repeated no-alloc calls differ"
    assert_attention_close(runs[0], regular.float().cpu().numpy(), q.dtype, f"{case}: no-alloc vs regular")
    assert_attention_close(runs[0], want, q.dtype, f"{case}: no-alloc vs oracle")
    assert capi.wait_timeouts(0) == 0
