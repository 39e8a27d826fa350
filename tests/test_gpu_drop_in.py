"""GPU: a caller written against DecodeKernels, unchanged (``import
decode_kernels as dk``), runs this library's kernels and matches the oracle --
through the wrapper with and without a preallocated workspace, and through
the raw torch op with the reference's schema."""

import pytest
import torch

import decode_kernels as dk
from decode_kernels.testing import make_paged_kv
from gpu_helpers import assert_attention_close, oracle_dense

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_reference_style_caller(dtype):
    lens = [1, 511, 512, 513, 0, 2000]
    kv = make_paged_kv(lens, 8, 128, 16, dtype, "cuda", layout="vllm", seed=3)
    q = torch.randn(len(lens), 32, 128, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda",
                    dtype=dtype)
    want = oracle_dense(q, kv)

    out = dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens)
    torch.cuda.synchronize()
    assert_attention_close(out, want, dtype, "decode_kernels.paged_attention_decode")

    ws = dk.alloc_workspace(len(lens), 32, 128, max(lens), "cuda")
    out2 = torch.full_like(q, float("nan"))
    dk.paged_attention_decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, max_seq_len=max(lens),
                              out=out2, workspace=ws)
    torch.cuda.synchronize()
    assert_attention_close(out2, want, dtype, "decode_kernels.paged_attention_decode (workspace)")
    out3 = torch.full_like(q, float("nan"))
    torch.ops.decode_kernels.paged_attention_decode(out3, q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens,
                                                    128**-0.5, max(lens), *ws)
    torch.cuda.synchronize()
    assert_attention_close(out3, want, dtype, "torch.ops.decode_kernels.paged_attention_decode")
