"""CPU: the vLLM integration's eligibility rules and plugin switches.

Eligible batches are pure decode on an fp16/bf16 cache laid out as vLLM 0.22
stores it ([2, num_blocks, block_size, num_kv_heads, head_size]); anything
else must fall back to FlashAttention (DecodeKernels
decode_kernels/vllm_patch.py:60-99 lists the same refusals).
"""

import logging
from types import SimpleNamespace

import pytest
import torch

vllm = pytest.importorskip("vllm")

from decodekernels_b200 import vllm_patch, vllm_plugin  # noqa: E402


def _case(**over):
    from vllm.v1.attention.backend import AttentionType

    n, hq, hkv, d = 3, 8, 2, 128
    impl = SimpleNamespace(attn_type=AttentionType.DECODER, dcp_world_size=1, kv_cache_dtype="auto",
                           alibi_slopes=None, logits_soft_cap=None, sliding_window=None, sinks=None, head_size=d,
                           num_heads=hq, num_kv_heads=hkv, scale=d**-0.5)
    meta = SimpleNamespace(max_query_len=1, use_cascade=False, causal=True, num_actual_tokens=n,
                           seq_lens=torch.ones(n, dtype=torch.int32), block_table=torch.zeros(n, 4, dtype=torch.int32),
                           max_seq_len=1)
    query = torch.zeros(n, hq, d, dtype=torch.bfloat16)
    kv_cache = torch.zeros(2, 10, 16, hkv, d, dtype=torch.bfloat16)
    output = torch.zeros(n, hq * d, dtype=torch.bfloat16)
    args = dict(impl=impl, query=query, kv_cache=kv_cache, attn_metadata=meta, output=output, output_scale=None,
                output_block_scale=None)
    for k, v in over.items():
        target, attr = k.split(".") if "." in k else (k, None)
        if attr is None:
            args[target] = v
        else:
            setattr(args[target], attr, v)
    return args


def test_pure_decode_is_eligible():
    assert vllm_patch._attention_eligible(**_case())


@pytest.mark.parametrize("over", [
    {"attn_metadata.max_query_len": 4},                  # prefill / mixed batch
    {"attn_metadata": None},                             # profiling run
    {"attn_metadata.use_cascade": True},
    {"impl.dcp_world_size": 2},                          # decode context parallelism
    {"impl.kv_cache_dtype": "fp8"},                     # fp8 needs a uint8 cache and the layer's scales
    {"impl.kv_cache_dtype": "fp8_e5m2", "kv_cache": torch.zeros(2, 10, 16, 2, 128, dtype=torch.uint8)},
    {"impl.alibi_slopes": torch.ones(8)},
    {"impl.logits_soft_cap": 30.0},
    {"impl.sliding_window": (127, 0)},
    {"impl.sinks": torch.zeros(8)},
    {"impl.head_size": 96},
    {"impl.num_heads": 32, "impl.num_kv_heads": 2},      # group 16 > 8
    {"attn_metadata.causal": False},
    {"output_scale": torch.ones(1)},
    {"query": torch.zeros(3, 8, 128, dtype=torch.float32)},
    {"kv_cache": torch.zeros(10, 16, 2, 256, dtype=torch.bfloat16)},  # not vLLM 0.22's [2, ...] cache
])
def test_refusals_fall_back(over):
    assert not vllm_patch._attention_eligible(**_case(**over))


def test_fp8_e4m3_cache_with_layer_scales_is_eligible():
    layer = SimpleNamespace(_k_scale_float=0.02, _v_scale_float=0.5)
    fp8 = torch.zeros(2, 10, 16, 2, 128, dtype=torch.uint8)
    for kvd in ("fp8", "fp8_e4m3"):
        assert vllm_patch._attention_eligible(**_case(**{"impl.kv_cache_dtype": kvd, "kv_cache": fp8}), layer=layer)
        assert vllm_patch._attention_eligible(
            **_case(**{"impl.kv_cache_dtype": kvd, "kv_cache": fp8.view(torch.float8_e4m3fn)}), layer=layer)
    # no layer / unusable scales / an fp8 query fall back
    assert not vllm_patch._attention_eligible(**_case(**{"impl.kv_cache_dtype": "fp8", "kv_cache": fp8}))
    bad = SimpleNamespace(_k_scale_float=0.0, _v_scale_float=1.0)
    assert not vllm_patch._attention_eligible(**_case(**{"impl.kv_cache_dtype": "fp8", "kv_cache": fp8}), layer=bad)
    q8 = torch.zeros(3, 8, 128, dtype=torch.float8_e4m3fn)
    assert not vllm_patch._attention_eligible(**_case(**{"impl.kv_cache_dtype": "fp8", "kv_cache": fp8,
                                                         "query": q8}), layer=layer)


def test_non_contiguous_output_falls_back():
    case = _case()
    case["output"] = torch.zeros(3, 2 * 8 * 128, dtype=torch.bfloat16)[:, ::2]
    assert not vllm_patch._attention_eligible(**case)


def test_plugin_is_a_no_op_unless_enabled(monkeypatch):
    calls = []
    monkeypatch.setattr(vllm_patch, "apply", lambda ops=None: calls.append(ops))
    monkeypatch.delenv("DECODE_KERNELS_VLLM", raising=False)
    vllm_plugin.register()
    assert calls == []
    monkeypatch.setenv("DECODE_KERNELS_VLLM", "1")
    monkeypatch.setenv("DECODE_KERNELS_OPS", "attention, rms_norm")
    vllm_plugin.register()
    assert calls == [["attention", "rms_norm"]]


def test_apply_without_gpu_leaves_vllm_alone(caplog):
    from vllm.v1.attention.backends.flash_attn import FlashAttentionImpl

    before = FlashAttentionImpl.forward
    if vllm_patch.dk_ops.is_available():
        pytest.skip("a GPU is visible; covered by the GPU test")
    with caplog.at_level(logging.WARNING, logger="decodekernels_b200.vllm"):
        vllm_patch.apply()
    assert FlashAttentionImpl.forward is before
    assert "unpatched" in caplog.text


def test_stats_reset():
    vllm_patch._STATS["attention_kernel_calls"] = 5
    vllm_patch.reset_stats()
    assert vllm_patch.stats() == {"attention_kernel_calls": 0, "attention_fallback_calls": 0}
