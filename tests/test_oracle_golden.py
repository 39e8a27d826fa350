"""CPU: pin the oracle against the reference's golden vectors.

The golden outputs come from running the reference's own
``paged_attention_reference`` / ``split_k_attention_reference`` on inputs
built by the reference's ``make_paged_kv`` (tests/golden/make_golden.py).
Here the inputs are rebuilt with this package's fixture builder (digests must
match) and the numpy oracle must reproduce the reference's outputs.
"""

import numpy as np
import pytest

from golden_cases import build, load_cases, outputs
from oracle import oracle

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_fixture_builder_reproduces_reference_inputs(case):
    build(case)  # asserts the sha256 digests of every input tensor


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_dense_oracle_matches_reference(case):
    q, kv = build(case)
    gold = outputs(case)
    got = oracle.paged_attention_dense(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale=case["scale"])
    if case["dtype"] == "float32":
        np.testing.assert_allclose(got, gold["dense"], atol=1e-5, rtol=1e-5)
    else:
        # The reference rounds its fp32 result to the input dtype.  fp32 sums in a
        # different order can land on the other side of a rounding boundary, so
        # allow exactly one ulp of that dtype (relative spacing 2^-8..2^-7 for
        # bf16, 2^-11..2^-10 for fp16) and require nearly all values bit-equal.
        ulp = 2.0**-7 if case["dtype"] == "bfloat16" else 2.0**-10
        rounded = oracle.round_to(got, case["dtype"])
        np.testing.assert_allclose(rounded, gold["dense"], atol=1e-7, rtol=ulp)
        assert np.mean(rounded != gold["dense"]) < 1e-2


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_split_oracle_matches_reference(case):
    q, kv = build(case)
    gold = outputs(case)
    for ps in case["partitions"]:
        out, tmp, m, s = oracle.split_k_attention(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens,
                                                  scale=case["scale"], partition_size=ps)
        np.testing.assert_allclose(out, gold[f"split_{ps}"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("case", [c for c in CASES if c["name"].startswith("merge_")], ids=lambda c: c["name"])
def test_split_equals_dense(case):
    """tests/test_reference.py:30-42: the partition / LSE merge equals dense attention."""
    q, kv = build(case)
    dense = oracle.paged_attention_dense(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    for ps in case["partitions"]:
        out = oracle.split_k_attention(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, partition_size=ps)[0]
        np.testing.assert_allclose(out, dense, atol=1e-5, rtol=1e-5)


def test_partition_statistics_layout():
    """Workspace row (seq*Hq + qh)*P + p holds partition p's (o, m, s); rows past the end stay unwritten."""
    case = next(c for c in CASES if c["name"] == "merge_d64_g4")
    q, kv = build(case)
    out, tmp, m, s = oracle.split_k_attention(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens,
                                              partition_size=64)
    lens = case["seq_lens"]
    assert tmp.shape == (len(lens), case["num_q_heads"], -(-max(lens) // 64), case["head_dim"])
    for si, L in enumerate(lens):
        live = -(-L // 64)
        assert np.isfinite(m[si, :, :live]).all() and np.isnan(m[si, :, live:]).all()
        assert (s[si, :, :live] >= 1.0 - 1e-6).all()  # the max term contributes exp(0) = 1
        merged = oracle.merge_partitions(tmp[si], m[si], s[si], live)
        np.testing.assert_allclose(merged, out[si], atol=1e-6, rtol=1e-6)


def test_empty_sequences_give_zeros():
    case = next(c for c in CASES if c["name"] == "empty_f16")
    q, kv = build(case)
    out = oracle.paged_attention_dense(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    assert not out[0].any() and not out[2].any()
    assert np.isfinite(out).all()


def test_round_to_matches_torch():
    import torch

    x = torch.randn(4096, dtype=torch.float32) * 10
    for dt, name in ((torch.bfloat16, "bfloat16"), (torch.float16, "float16")):
        np.testing.assert_array_equal(oracle.round_to(x.numpy(), name), x.to(dt).float().numpy())
