"""Helpers shared by the GPU parity tests: run the CUDA path through the C ABI
and compare with the CPU oracle under the tolerances of the spec."""

from __future__ import annotations

import numpy as np
import torch

from decodekernels_b200 import capi
from oracle import oracle

# The reference's kernel-test tolerances (tests/test_kernels.py:25 of DecodeKernels) ...
ATTN_TOL = {torch.float16: dict(atol=3e-3, rtol=1e-2), torch.bfloat16: dict(atol=2e-2, rtol=2e-2)}
# ... and the north-star bound for fp16/bf16 against both oracles.
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def alloc_ws(num_seqs, num_q_heads, head_dim, parts, device, fill=float("nan")):
    tmp = torch.full((num_seqs, num_q_heads, parts, head_dim), fill, dtype=torch.float32, device=device)
    ml = torch.full((num_seqs, num_q_heads, parts), fill, dtype=torch.float32, device=device)
    es = torch.full((num_seqs, num_q_heads, parts), fill, dtype=torch.float32, device=device)
    return tmp, ml, es


def run_capi(q, kv, scale=None, max_seq_len=None, partition_size=0, force_simt=False, workspace="auto", out=None,
             counters=False, flags=0):
    """Call dk_paged_attention_decode; returns (out, workspace, plan).  With
    ``counters`` the workspace gets zeroed merge counters (single launch)."""
    n, hq, d = q.shape
    scale = d**-0.5 if scale is None else scale
    if max_seq_len is None:
        max_seq_len = int(kv.seq_lens.max().item()) if n else 0
    if out is None:
        out = torch.full_like(q, float("nan"))
    if workspace == "auto":
        if partition_size:
            parts = max(1, -(-max_seq_len // partition_size))
        else:
            parts = capi.num_partitions(n, kv.k_cache.shape[2], d, kv.k_cache.shape[1], max_seq_len)
        workspace = alloc_ws(n, hq, d, parts, q.device)
        if counters:
            workspace = (*workspace, torch.zeros(n * kv.k_cache.shape[2], dtype=torch.int32, device=q.device))
    plan = capi.plan(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale, max_seq_len, out, workspace,
                     partition_size, force_simt, flags)
    capi.decode(q, kv.k_cache, kv.v_cache, kv.block_tables, kv.seq_lens, scale, max_seq_len, out, workspace,
                partition_size, force_simt, flags=flags)
    torch.cuda.synchronize()
    return out, workspace, plan


def oracle_dense(q, kv, scale=None):
    return oracle.paged_attention_dense(q.cpu(), kv.k_cache.cpu(), kv.v_cache.cpu(), kv.block_tables.cpu().numpy(),
                                        kv.seq_lens.cpu().numpy(), scale=scale)


def assert_attention_close(got: torch.Tensor, want: np.ndarray, dtype, what: str = "") -> None:
    """Kernel output vs a float32 oracle: reference tolerance and north-star bounds."""
    g = got.float().cpu().numpy()
    assert np.isfinite(g).all(), f"{what}: non-finite output"
    err = np.abs(g - want)
    assert err.max() <= MAX_ABS, f"{what}: max-abs {err.max():.3e} > {MAX_ABS}"
    assert err.mean() <= MEAN_ABS, f"{what}: mean-abs {err.mean():.3e} > {MEAN_ABS}"
    tol = ATTN_TOL[dtype]
    np.testing.assert_allclose(g, want, atol=tol["atol"], rtol=tol["rtol"], err_msg=what)


def assert_workspace_matches(ws, kv, q, partition_size, scale=None, what=""):
    """Live workspace rows hold the oracle's per-partition (o, m, s); rows of
    partitions past each sequence's end are untouched (still NaN)."""
    tmp, ml, es = (t.cpu().numpy() for t in ws)
    P = tmp.shape[2]
    _, o_ref, m_ref, s_ref = oracle.split_k_attention(q.cpu(), kv.k_cache.cpu(), kv.v_cache.cpu(),
                                                      kv.block_tables.cpu().numpy(), kv.seq_lens.cpu().numpy(),
                                                      scale=scale, partition_size=partition_size, num_partitions=P)
    lens = kv.seq_lens.cpu().numpy()
    for s, L in enumerate(lens):
        live = min(-(-int(L) // partition_size), P) if L > 0 else 0
        assert np.isnan(ml[s, :, live:]).all() and np.isnan(es[s, :, live:]).all(), f"{what}: seq {s} wrote past end"
        assert np.isnan(tmp[s, :, live:]).all(), f"{what}: seq {s} wrote tmp_out past end"
        if live == 0:
            continue
        np.testing.assert_allclose(ml[s, :, :live], m_ref[s, :, :live], atol=2e-2, rtol=1e-2, err_msg=f"{what} m")
        np.testing.assert_allclose(es[s, :, :live], s_ref[s, :, :live], atol=2e-2, rtol=2e-2, err_msg=f"{what} s")
        np.testing.assert_allclose(tmp[s, :, :live], o_ref[s, :, :live], atol=2e-2, rtol=2e-2, err_msg=f"{what} o")


def fp8_caches(kv, layout, k_scale, v_scale):
    """e4m3 copies (uint8) of a 16-bit paged cache in the same layout -- one
    interleaved K|V buffer for the "vllm" layout, so the fused TMA map is used
    -- quantised as sat_e4m3(x / scale)."""
    nb, bs, h, d = kv.k_cache.shape
    if layout == "vllm":
        buf = torch.empty(nb, h, bs, 2 * d, dtype=torch.uint8, device=kv.k_cache.device)
        k8, v8 = buf.transpose(1, 2).split(d, dim=-1)
    elif layout == "hnd":
        k8 = torch.empty(nb, h, bs, d, dtype=torch.uint8, device=kv.k_cache.device).transpose(1, 2)
        v8 = torch.empty(nb, h, bs, d, dtype=torch.uint8, device=kv.k_cache.device).transpose(1, 2)
    else:
        k8 = torch.empty(nb, bs, h, d, dtype=torch.uint8, device=kv.k_cache.device)
        v8 = torch.empty_like(k8)
    for dst, src, s in ((k8, kv.k_cache, k_scale), (v8, kv.v_cache, v_scale)):
        q8 = (src.float() / s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
        dst.copy_(q8)
    return k8, v8


def oracle_dense_fp8(q, kv, k8, v8, k_scale, v_scale, scale=None):
    """The oracle on the dequantised e4m3 caches (code * scale)."""
    from oracle import cache_write as cw

    kd = cw.e4m3_decode(k8.cpu().numpy()) * np.float32(k_scale)
    vd = cw.e4m3_decode(v8.cpu().numpy()) * np.float32(v_scale)
    return oracle.paged_attention_dense(q.cpu(), kd, vd, kv.block_tables.cpu().numpy(), kv.seq_lens.cpu().numpy(),
                                        scale=scale)
