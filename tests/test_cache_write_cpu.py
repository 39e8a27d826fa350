"""CPU: the paged-KV write oracle (oracle/cache_write.py) and the C ABI's
argument checks for dk_reshape_and_cache (no compute calls without a GPU).

The e4m3 encoder is pinned to torch's independent float8_e4m3fn conversion
(clamped to +-448, the saturating convention) on random values and on every
code boundary, tie, subnormal and special value."""

import ctypes

import numpy as np
import pytest
import torch

from decodekernels_b200 import capi
from oracle import cache_write as cw


def _torch_e4m3(x: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.asarray(x, dtype=np.float32))
    t = torch.where(torch.isnan(t), t, t.clamp(-cw.E4M3_MAX, cw.E4M3_MAX))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def test_decode_table():
    codes = np.arange(256, dtype=np.uint8)
    vals = cw.e4m3_decode(codes)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(vals), np.isnan(ref))
    ok = ~np.isnan(vals)
    assert np.array_equal(vals[ok], ref[ok])
    assert vals[0x7E] == 448.0 and vals[0x01] == 2.0**-9


def test_encode_matches_torch_on_every_boundary():
    finite = cw.e4m3_decode(np.arange(127, dtype=np.uint8)).astype(np.float64)
    mids = (finite[:-1] + finite[1:]) / 2  # exact ties
    probes = np.concatenate([finite, mids, np.nextafter(mids, 0), np.nextafter(mids, 1e9), [448.0, 449.0, 463.9, 464.0,
                             465.0, 1e6, np.inf, 2.0**-10, 2.0**-11, 1e-30, 0.0]])
    x = np.concatenate([probes, -probes, [np.nan]]).astype(np.float32)
    got = cw.e4m3_encode(x)
    want = _torch_e4m3(x)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], want[~nan])
    assert (got[nan] & 0x7F) == 0x7F


def test_encode_matches_torch_random():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000) * s for s in (1e-3, 0.1, 1.0, 30.0, 1000.0)]).astype(np.float32)
    assert np.array_equal(cw.e4m3_encode(x), _torch_e4m3(x))


def test_quantize_divides_in_float32():
    x = np.array([1.0, 3.0, -7.5, 0.3], dtype=np.float32)
    scale = np.float32(0.37)
    assert np.array_equal(cw.quantize(x, scale), cw.e4m3_encode((x / scale).astype(np.float32)))


def test_oracle_scatter_skips_padding_and_out_of_range():
    rng = np.random.default_rng(1)
    T, H, D, nb, bs = 6, 2, 8, 3, 4
    k = rng.standard_normal((T, H, D)).astype(np.float32)
    v = rng.standard_normal((T, H, D)).astype(np.float32)
    kc = np.zeros((nb, bs, H, D), np.float32)
    vc = np.zeros_like(kc)
    slots = np.array([0, 5, -1, 11, 12, 7])
    cw.reshape_and_cache(k, v, kc, vc, slots)
    assert np.array_equal(kc[0, 0], k[0]) and np.array_equal(vc[1, 1], v[1]) and np.array_equal(kc[2, 3], k[3])
    assert np.array_equal(kc[1, 3], k[5])
    written = {(0, 0), (1, 1), (2, 3), (1, 3)}
    for b in range(nb):
        for o in range(bs):
            if (b, o) not in written:
                assert not kc[b, o].any() and not vc[b, o].any()


def _args(cache=torch.bfloat16, **over):
    """Struct for CPU tensors (shapes / strides / pointers only); ``over`` sets fields."""
    T, H, D, nb, bs = 4, 2, 64, 8, 16
    key = torch.zeros(T, H, D, dtype=torch.bfloat16)
    kc = torch.zeros(nb, bs, H, D, dtype=cache)
    slots = torch.zeros(T, dtype=torch.int64)
    a = capi.make_cache_write_args(key, key, kc, kc, slots)
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("cache,override,msg", [
    (torch.bfloat16, dict(dtype=7), "float16 or bfloat16"),
    (torch.bfloat16, dict(dtype=0), "cache dtype"),
    (torch.bfloat16, dict(num_tokens=-1), "num_tokens"),
    (torch.bfloat16, dict(head_dim=0), "positive"),
    (torch.uint8, dict(k_scale=0.0), "scales"),
    (torch.uint8, dict(v_scale=float("inf")), "scales"),
    (torch.bfloat16, dict(key_stride_head=-8), "negative stride"),
])
def test_cache_write_validation(cache, override, msg):
    a = _args(cache, **override)
    assert capi.load().dk_reshape_and_cache(ctypes.byref(a), None) == 1
    assert msg in capi.last_error()


def test_cache_write_args_layout():
    a = _args(torch.uint8, k_scale=0.5)
    assert a.cache_dtype == capi.DK_DTYPE_FP8_E4M3 and a.dtype == capi.DK_DTYPE_BFLOAT16 and a.k_scale == 0.5
    assert (a.num_tokens, a.num_kv_heads, a.head_dim, a.num_blocks, a.block_size) == (4, 2, 64, 8, 16)
    assert (a.k_stride_block, a.k_stride_token, a.k_stride_head) == (16 * 2 * 64, 2 * 64, 64)
    # zero tokens is a no-op that touches nothing
    z = _args(num_tokens=0)
    assert capi.load().dk_reshape_and_cache(ctypes.byref(z), None) == 0
