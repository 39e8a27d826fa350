"""GPU: the patched vLLM FlashAttentionImpl.forward runs this library's
kernels on a vLLM 0.22 KV cache ([2, num_blocks, block_size, num_kv_heads,
head_size], both stride orders vLLM uses) and matches the oracle."""

from types import SimpleNamespace

import pytest
import torch

import decodekernels_b200 as dk
from decodekernels_b200.testing import PagedKV
from gpu_helpers import assert_attention_close, oracle_dense

vllm = pytest.importorskip("vllm")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not dk.is_available(), reason="needs a CUDA GPU and the built native library"),
]


@pytest.mark.parametrize("stride_order", ["nhd", "hnd"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_patched_forward_decodes_on_vllm_cache(stride_order, dtype):
    from vllm.v1.attention.backend import AttentionType
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl

    from decodekernels_b200 import vllm_patch

    vllm_patch.apply(["attention"])
    vllm_patch.reset_stats()

    n, hq, hkv, d, bs = 5, 32, 8, 128, 16
    lens = [1, 700, 2049, 64, 3000]
    nb = sum(-(-L // bs) for L in lens) + 4
    g = torch.Generator(device="cuda").manual_seed(7)
    if stride_order == "nhd":
        kv_cache = torch.randn(2, nb, bs, hkv, d, generator=g, device="cuda", dtype=dtype)
    else:  # physical [2, blocks, heads, bs, D] viewed as vLLM's logical shape
        kv_cache = torch.randn(2, nb, hkv, bs, d, generator=g, device="cuda", dtype=dtype).transpose(2, 3)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(8)).to(torch.int32)
    width = max(-(-L // bs) for L in lens)
    table = torch.zeros(n, width, dtype=torch.int32)
    off = 0
    for i, L in enumerate(lens):
        k = -(-L // bs)
        table[i, :k] = perm[off:off + k]
        off += k
    impl = SimpleNamespace(attn_type=AttentionType.DECODER, dcp_world_size=1, kv_cache_dtype="auto",
                           alibi_slopes=None, logits_soft_cap=None, sliding_window=None, sinks=None, head_size=d,
                           num_heads=hq, num_kv_heads=hkv, scale=d**-0.5)
    meta = SimpleNamespace(max_query_len=1, use_cascade=False, causal=True, num_actual_tokens=n,
                           seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"), block_table=table.cuda(),
                           max_seq_len=max(lens))
    query = torch.randn(n, hq, d, generator=g, device="cuda", dtype=dtype)
    output = torch.full((n, hq * d), float("nan"), device="cuda", dtype=dtype)
    ret = FlashAttentionImpl.forward(impl, None, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    assert ret is output
    assert vllm_patch.stats()["attention_kernel_calls"] == 1
    k_cache, v_cache = kv_cache.unbind(0)
    ref = oracle_dense(query, PagedKV(k_cache, v_cache, meta.block_table, meta.seq_lens, bs))
    assert_attention_close(output.view(n, hq, d), ref, dtype, f"vllm {stride_order}")


@pytest.mark.parametrize("stride_order", ["nhd", "hnd"])
def test_patched_forward_decodes_fp8_vllm_cache(stride_order):
    """vLLM's fp8 (e4m3) cache -- uint8 codes written as x / scale -- with the
    layer's per-tensor scales decodes here and matches the oracle on the
    dequantised cache."""
    from vllm.v1.attention.backend import AttentionType
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl

    from decodekernels_b200 import vllm_patch
    from gpu_helpers import oracle_dense_fp8

    vllm_patch.apply(["attention"])
    vllm_patch.reset_stats()
    dtype, n, hq, hkv, d, bs = torch.bfloat16, 4, 16, 2, 128, 16
    ks, vs = 0.02, 0.03
    lens = [5, 900, 2049, 64]
    nb = sum(-(-L // bs) for L in lens) + 4
    g = torch.Generator(device="cuda").manual_seed(9)
    if stride_order == "nhd":
        vals = torch.randn(2, nb, bs, hkv, d, generator=g, device="cuda")
        kv_cache = torch.empty(2, nb, bs, hkv, d, dtype=torch.uint8, device="cuda")
    else:
        vals = torch.randn(2, nb, hkv, bs, d, generator=g, device="cuda").transpose(2, 3)
        kv_cache = torch.empty(2, nb, hkv, bs, d, dtype=torch.uint8, device="cuda").transpose(2, 3)
    kv_cache[0].copy_((vals[0] / ks).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8))
    kv_cache[1].copy_((vals[1] / vs).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8))
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(10)).to(torch.int32)
    table = torch.zeros(n, max(-(-L // bs) for L in lens), dtype=torch.int32)
    off = 0
    for i, L in enumerate(lens):
        k = -(-L // bs)
        table[i, :k] = perm[off:off + k]
        off += k
    impl = SimpleNamespace(attn_type=AttentionType.DECODER, dcp_world_size=1, kv_cache_dtype="fp8",
                           alibi_slopes=None, logits_soft_cap=None, sliding_window=None, sinks=None, head_size=d,
                           num_heads=hq, num_kv_heads=hkv, scale=d**-0.5)
    layer = SimpleNamespace(_k_scale_float=ks, _v_scale_float=vs)
    meta = SimpleNamespace(max_query_len=1, use_cascade=False, causal=True, num_actual_tokens=n,
                           seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"), block_table=table.cuda(),
                           max_seq_len=max(lens))
    query = torch.randn(n, hq, d, generator=g, device="cuda", dtype=dtype)
    output = torch.full((n, hq * d), float("nan"), device="cuda", dtype=dtype)
    ret = FlashAttentionImpl.forward(impl, layer, query, None, None, kv_cache, meta, output)
    torch.cuda.synchronize()
    assert ret is output and vllm_patch.stats()["attention_kernel_calls"] == 1
    k8, v8 = kv_cache.unbind(0)
    kv = PagedKV(k8, v8, meta.block_table, meta.seq_lens, bs)
    assert_attention_close(output.view(n, hq, d), oracle_dense_fp8(query, kv, k8, v8, ks, vs), dtype,
                           f"vllm fp8 {stride_order}")


def test_patched_forward_under_cuda_graph_capture():
    """vLLM's full-cudagraph mode: the forward is captured with max_seq_len =
    the model's maximum length and replayed after seq_lens and block_table
    were refreshed in place (longer and shorter sequences, new pages); every
    replay matches the oracle."""
    from vllm.v1.attention.backend import AttentionType
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl

    from decodekernels_b200 import vllm_patch

    vllm_patch.apply(["attention"])
    vllm_patch.reset_stats()
    dtype, n, hq, hkv, d, bs, max_model_len = torch.float16, 6, 16, 4, 128, 16, 4096
    nb = n * max_model_len // bs + 4
    g = torch.Generator(device="cuda").manual_seed(11)
    kv_cache = torch.randn(2, nb, bs, hkv, d, generator=g, device="cuda", dtype=dtype)
    width = max_model_len // bs
    seq_lens = torch.zeros(n, dtype=torch.int32, device="cuda")
    block_table = torch.zeros(n, width, dtype=torch.int32, device="cuda")
    query = torch.zeros(n, hq, d, device="cuda", dtype=dtype)
    output = torch.zeros(n, hq * d, device="cuda", dtype=dtype)
    impl = SimpleNamespace(attn_type=AttentionType.DECODER, dcp_world_size=1, kv_cache_dtype="auto",
                           alibi_slopes=None, logits_soft_cap=None, sliding_window=None, sinks=None, head_size=d,
                           num_heads=hq, num_kv_heads=hkv, scale=d**-0.5)
    meta = SimpleNamespace(max_query_len=1, use_cascade=False, causal=True, num_actual_tokens=n, seq_lens=seq_lens,
                           block_table=block_table, max_seq_len=max_model_len)

    def refresh(lens, seed):
        perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed)).to(torch.int32)
        table = torch.zeros(n, width, dtype=torch.int32)
        off = 0
        for i, L in enumerate(lens):
            k = -(-L // bs)
            table[i, :k] = perm[off:off + k]
            off += k
        block_table.copy_(table)
        seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
        query.copy_(torch.randn(n, hq, d, generator=torch.Generator(device="cuda").manual_seed(seed), device="cuda"))

    refresh([3, 17, 100, 64, 5, 1], 1)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up outside the graph, as vLLM does
        FlashAttentionImpl.forward(impl, None, query, None, None, kv_cache, meta, output)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        FlashAttentionImpl.forward(impl, None, query, None, None, kv_cache, meta, output)
    assert vllm_patch.stats()["attention_kernel_calls"] == 2  # the captured call ran here too
    assert vllm_patch.stats()["attention_fallback_calls"] == 0
    for lens, seed in (([4096, 1, 0, 2049, 513, 3000], 2), ([7, 4000, 1500, 0, 64, 65], 3)):
        refresh(lens, seed)
        output.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        k_cache, v_cache = kv_cache.unbind(0)
        ref = oracle_dense(query, PagedKV(k_cache, v_cache, block_table, seq_lens, bs))
        assert_attention_close(output.view(n, hq, d), ref, dtype, f"captured, lens {lens}")
    del graph
