"""CPU: the C restatement of the oracle (used for the timed CPU baseline and
large parity checks) agrees with the numpy oracle, which the golden vectors pin."""

import numpy as np
import pytest
import torch

from golden_cases import build, load_cases
from oracle import native, oracle

HALF = [c for c in load_cases() if c["dtype"] != "float32"]


@pytest.mark.parametrize("case", HALF, ids=[c["name"] for c in HALF])
def test_c_oracle_matches_numpy_oracle(case):
    q, kv = build(case)
    want = oracle.paged_attention_dense(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale=case["scale"])
    got = native.dense_c(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale=case["scale"])
    np.testing.assert_allclose(got, want, atol=2e-5, rtol=2e-5)


def test_c_oracle_half_conversion_is_exact():
    x = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.float16).reshape(1, 1, 1, 65536)
    # one "token" whose K row is every fp16 bit pattern: q = e_i picks element i
    assert x.numel() == 65536
    bits = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16)
    ref = bits.view(torch.float16).float()
    from oracle.native import DkOracleArgs  # noqa: F401  (struct layout import check)
    finite = torch.isfinite(ref)
    # run 64-wide chunks through the oracle as V rows with a single token (softmax weight 1)
    vals = bits.view(torch.float16)[finite][: 64 * 512].reshape(512, 1, 1, 64)
    k = torch.zeros_like(vals)
    q = torch.zeros(1, 1, 64, dtype=torch.float16)
    for blk in range(0, 512, 64):
        v = vals[blk:blk + 64]
        bt = torch.arange(64, dtype=torch.int32).reshape(64, 1)
        sl = torch.ones(64, dtype=torch.int32)
        qq = q.expand(64, 1, 64).contiguous()
        out = native.dense_c(qq, k[blk:blk + 64], v, bt, sl, scale=1.0)
        np.testing.assert_array_equal(out[:, 0, :], v[:, 0, 0, :].float().numpy())


def test_c_oracle_threads():
    assert native.max_threads() >= 1


def test_c_oracle_head_split_is_bit_identical():
    # More threads than (sequence, KV head) pairs: the work is split per query
    # head, which must not change a single bit of the result.
    case = next(c for c in HALF if c["name"] == "c1")
    q, kv = build(case)
    args = (q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    one, many = {}, {}
    a = native.dense_c(*args, scale=case["scale"], num_threads=1, info=one)
    b = native.dense_c(*args, scale=case["scale"], num_threads=64, info=many)
    assert one == {"threads_used": 1, "units": 4 * 8}
    assert many["units"] == 4 * 32 and many["threads_used"] >= 1
    np.testing.assert_array_equal(a, b)
