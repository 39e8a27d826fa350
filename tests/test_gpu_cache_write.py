"""GPU: the paged-KV write (dk_reshape_and_cache / dk.reshape_and_cache)
against the CPU oracle (bit-exact, 16-bit and FP8 e4m3 caches, every decode
layout, padding slots, unaligned rows), against vLLM's own
reshape_and_cache_flash when vLLM's kernels load on this machine, and end to
end: tokens written by it decode like a cache built directly."""

import numpy as np
import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200 import capi
from decodekernels_b200.testing import make_paged_kv
from gpu_helpers import assert_attention_close, oracle_dense
from oracle import cache_write as cw

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]


def _caches(nb, bs, H, D, dtype, layout):
    """Two caches [nb, bs, H, D] in a decode layout, filled with a sentinel."""
    fill = 0x5A if dtype in (torch.uint8, torch.float8_e4m3fn) else 7.0
    if layout == "nhd":
        kc = torch.empty(nb, bs, H, D, dtype=dtype, device="cuda")
        vc = torch.empty_like(kc)
    elif layout == "hnd":
        kc = torch.empty(nb, H, bs, D, dtype=dtype, device="cuda").transpose(1, 2)
        vc = torch.empty(nb, H, bs, D, dtype=dtype, device="cuda").transpose(1, 2)
    else:  # vLLM 0.22: [2, blocks, bs, H, D] split by unbind(0)
        kc, vc = torch.empty(2, nb, bs, H, D, dtype=dtype, device="cuda").unbind(0)
    for c in (kc, vc):
        c.view(torch.uint8).fill_(fill) if dtype == torch.float8_e4m3fn else c.fill_(fill)
    return kc, vc


def _np(t):
    if t.dtype in (torch.uint8, torch.float8_e4m3fn):
        return t.view(torch.uint8).cpu().numpy()
    return t.float().cpu().numpy()


def _inputs(T, H, D, dtype, nb, bs, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    key = torch.randn(T, H, D, generator=g, device="cuda", dtype=torch.float32).mul_(3.0).to(dtype)
    value = torch.randn(T, H, D, generator=g, device="cuda", dtype=torch.float32).mul_(3.0).to(dtype)
    gc = torch.Generator().manual_seed(seed)
    slots = torch.randperm(nb * bs, generator=gc)[:T].to(torch.int64)
    slots[::5] = -1  # padding tokens
    return key, value, slots.cuda()


def _oracle(key, value, kc0, vc0, slots, k_scale, v_scale, fp8):
    kc, vc = _np(kc0).copy(), _np(vc0).copy()
    k = key.float().cpu().numpy()
    v = value.float().cpu().numpy()
    if fp8:
        kc, vc = kc.astype(np.uint8), vc.astype(np.uint8)
    cw.reshape_and_cache(k, v, kc, vc, slots.cpu().numpy(), k_scale, v_scale, fp8=fp8)
    return kc, vc


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("cache", ["same", torch.uint8, torch.float8_e4m3fn])
@pytest.mark.parametrize("layout", ["nhd", "hnd", "vllm"])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_matches_oracle_bit_exact(dtype, cache, layout, D):
    cache_dtype = dtype if cache == "same" else cache
    fp8 = cache != "same"
    H, nb, bs, T = 4, 24, 16, 150
    key, value, slots = _inputs(T, H, D, dtype, nb, bs, seed=D)
    kc, vc = _caches(nb, bs, H, D, cache_dtype, layout)
    k_scale, v_scale = (0.37, 2.5) if fp8 else (1.0, 1.0)
    want_k, want_v = _oracle(key, value, kc, vc, slots, k_scale, v_scale, fp8)
    dk.reshape_and_cache(key, value, kc, vc, slots, k_scale, v_scale)
    torch.cuda.synchronize()
    assert np.array_equal(_np(kc), want_k)
    assert np.array_equal(_np(vc), want_v)


@pytest.mark.parametrize("fp8", [False, True])
def test_unaligned_rows_take_the_element_path(fp8):
    """Rows that do not start on 16 bytes (a key view offset by one element)."""
    dtype, H, D, nb, bs, T = torch.bfloat16, 2, 64, 8, 16, 40
    big = torch.randn(T * H * D + 1, device="cuda", dtype=torch.float32).to(dtype)
    key = big[1:].view(T, H, D)
    value = torch.randn(T, H, D, device="cuda", dtype=torch.float32).to(dtype)
    slots = torch.arange(T, dtype=torch.int64, device="cuda") * 3 % (nb * bs)
    kc, vc = _caches(nb, bs, H, D, torch.uint8 if fp8 else dtype, "nhd")
    want_k, want_v = _oracle(key, value, kc, vc, slots, 0.5, 0.5, fp8)
    capi.reshape_and_cache(key, value, kc, vc, slots, 0.5, 0.5)
    torch.cuda.synchronize()
    assert np.array_equal(_np(kc), want_k) and np.array_equal(_np(vc), want_v)


def test_saturation_and_specials():
    """Values past +-448 * scale saturate; NaN stays NaN; -0 keeps its sign."""
    H, D, nb, bs = 1, 64, 2, 16
    key = torch.zeros(3, H, D, dtype=torch.float16, device="cuda")
    key[0, 0, :8] = torch.tensor([1e4, -1e4, 448.0, 464.0, 465.0, float("nan"), -0.0, 2.0**-10])
    value = key.clone()
    slots = torch.tensor([0, 1, -7], dtype=torch.int64, device="cuda")
    kc, vc = _caches(nb, bs, H, D, torch.uint8, "nhd")
    want_k, _ = _oracle(key, value, kc, vc, slots, 1.0, 1.0, True)
    dk.reshape_and_cache(key, value, kc, vc, slots, 1.0, 1.0)
    torch.cuda.synchronize()
    got = _np(kc)
    assert list(got[0, 0, 0, :5]) == [0x7E, 0xFE, 0x7E, 0x7E, 0x7E]
    assert got[0, 0, 0, 5] & 0x7F == 0x7F and got[0, 0, 0, 6] == 0x80 and got[0, 0, 0, 7] == 0x00
    got[0, 0, 0, 5] &= 0x7F  # the NaN's sign bit is not specified
    want_k[0, 0, 0, 5] &= 0x7F
    assert np.array_equal(got, want_k)


def _vllm_cache_op():
    try:
        import vllm._custom_ops  # noqa: F401  (loads vLLM's CUDA kernels)

        return torch.ops._C_cache_ops.reshape_and_cache_flash
    except Exception:
        return None


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("layout", ["nhd", "vllm"])
def test_matches_vllm_kernel(dtype, fp8, layout):
    op = _vllm_cache_op()
    if op is None:
        pytest.skip("vLLM's CUDA kernels do not load here")
    H, D, nb, bs, T = 8, 128, 64, 16, 300
    key, value, slots = _inputs(T, H, D, dtype, nb, bs, seed=7)
    cache_dtype = torch.uint8 if fp8 else dtype
    ours_k, ours_v = _caches(nb, bs, H, D, cache_dtype, layout)
    ref_k, ref_v = _caches(nb, bs, H, D, cache_dtype, layout)
    k_scale, v_scale = (0.61, 1.9) if fp8 else (1.0, 1.0)
    dk.reshape_and_cache(key, value, ours_k, ours_v, slots, k_scale, v_scale)
    op(key, value, ref_k, ref_v, slots, "fp8" if fp8 else "auto",
       torch.tensor(k_scale, dtype=torch.float32, device="cuda"), torch.tensor(v_scale, dtype=torch.float32,
                                                                                device="cuda"))
    torch.cuda.synchronize()
    for ours, ref in ((ours_k, ref_k), (ours_v, ref_v)):
        if not fp8:
            assert torch.equal(ours, ref)
            continue
        # vLLM may build its division x / scale with fast math: allow a
        # neighbouring code on a handful of elements, report how many
        a = ours.view(torch.uint8).cpu().numpy().astype(np.int16)
        b = ref.view(torch.uint8).cpu().numpy().astype(np.int16)
        diff = a != b
        assert diff.mean() <= 1e-3, f"{int(diff.sum())} of {diff.size} codes differ from vLLM's"
        assert np.all(np.abs(a - b)[diff] == 1)


@pytest.mark.parametrize("layout", ["nhd", "vllm"])
def test_written_tokens_decode_like_a_built_cache(layout):
    """Write every token of a paged cache through reshape_and_cache into an
    empty cache with the same block tables; the decode output is identical."""
    dtype = torch.bfloat16
    lens = [1, 300, 77, 1024]
    kv = make_paged_kv(lens, 2, 128, 16, dtype, "cuda", layout=layout, seed=3)
    kc, vc = _caches(kv.k_cache.shape[0], 16, 2, 128, dtype, layout)
    keys, values, slots = [], [], []
    bt = kv.block_tables.cpu()
    for s, L in enumerate(lens):
        for t in range(L):
            b = int(bt[s, t // 16])
            keys.append(kv.k_cache[b, t % 16])
            values.append(kv.v_cache[b, t % 16])
            slots.append(b * 16 + t % 16)
    key = torch.stack(keys)
    value = torch.stack(values)
    dk.reshape_and_cache(key, value, kc, vc, torch.tensor(slots, dtype=torch.int64, device="cuda"))
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn(len(lens), 8, 128, generator=g, device="cuda", dtype=dtype)
    want = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    got = dk.paged_attention_decode(q, kc, vc, kv.block_tables, kv.seq_lens)
    assert torch.equal(got, want)
    assert_attention_close(got, oracle_dense(q, kv), dtype, "written cache")
