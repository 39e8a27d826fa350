"""ctypes access to the compiled checkers.  TEST INFRASTRUCTURE, NOT PRODUCT.

* ``dense_c(...)``        the C restatement of the reference's dense oracle
                          (oracle/paged_attention_cpu.c), multithreaded;
* ``reference_kernel(...)`` the reference's own CUDA kernels built from its
                          source tree (oracle/_ref/libdk_ref_kernel.so), run on
                          the same device tensors as this library.

Only tests/, __graft_entry__.smoke() and bench.py use it -- bench.py as the
checker of its outputs before timing, as the timed CPU baseline, and to time
the reference's own kernel beside this library's for comparison.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "libdk_oracle.so"
REF_LIB = HERE / "_ref" / "libdk_ref_kernel.so"


class DkOracleArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("q_stride_seq", ctypes.c_int64),
        ("q_stride_head", ctypes.c_int64),
        ("k_stride_block", ctypes.c_int64),
        ("k_stride_token", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("v_stride_block", ctypes.c_int64),
        ("v_stride_token", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("bt_stride", ctypes.c_int64),
        ("num_seqs", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("num_threads", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("threads_used", ctypes.c_int32),
        ("units", ctypes.c_int32),
    ]


class DkRefArgs(ctypes.Structure):
    _fields_ = [
        ("out", ctypes.c_void_p),
        ("q", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("tmp_out", ctypes.c_void_p),
        ("max_logits", ctypes.c_void_p),
        ("exp_sums", ctypes.c_void_p),
        ("q_stride_seq", ctypes.c_int64),
        ("q_stride_head", ctypes.c_int64),
        ("out_stride_seq", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("k_stride_block", ctypes.c_int64),
        ("k_stride_token", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("v_stride_block", ctypes.c_int64),
        ("v_stride_token", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("bt_stride", ctypes.c_int64),
        ("num_seqs", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("max_partitions", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
    ]


_oracle = None
_ref = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            from . import build

            build.build_oracle()
        lib = ctypes.CDLL(str(ORACLE_LIB))
        lib.dk_oracle_paged_attention.argtypes = [ctypes.POINTER(DkOracleArgs)]
        lib.dk_oracle_paged_attention.restype = ctypes.c_int
        lib.dk_oracle_max_threads.restype = ctypes.c_int
        _oracle = lib
    return _oracle


def have_reference_kernel() -> bool:
    return REF_LIB.exists()


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(str(REF_LIB))
        lib.dk_ref_paged_attention_decode.argtypes = [ctypes.POINTER(DkRefArgs), ctypes.c_void_p]
        lib.dk_ref_paged_attention_decode.restype = ctypes.c_int
        _ref = lib
    return _ref


def _dtype_code(t) -> int:
    import torch

    return {torch.float16: 0, torch.bfloat16: 1}[t.dtype]


def dense_c(q, k_cache, v_cache, block_tables, seq_lens, scale=None, num_threads: int = 0,
            info: dict | None = None) -> np.ndarray:
    """Dense attention on the CPU through the C oracle.  Inputs are CPU torch
    tensors (fp16/bf16 q and caches, any strides); returns float32 numpy
    ``[num_seqs, Hq, D]``.  ``num_threads`` > 0 sets the OpenMP team size
    (0: OpenMP's default, which OMP_NUM_THREADS controls); ``info`` receives
    ``threads_used`` and ``units`` (parallel work units)."""
    import torch

    n, hq, d = q.shape
    scale = d**-0.5 if scale is None else scale
    bt = block_tables.to(torch.int32)
    sl = seq_lens.to(torch.int32).contiguous()
    out = np.zeros((n, hq, d), dtype=np.float32)
    a = DkOracleArgs()
    a.q, a.k_cache, a.v_cache = q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr()
    a.block_tables, a.seq_lens = bt.data_ptr(), sl.data_ptr()
    a.out = out.ctypes.data
    a.q_stride_seq, a.q_stride_head = q.stride(0), q.stride(1)
    a.k_stride_block, a.k_stride_token, a.k_stride_head = k_cache.stride()[:3]
    a.v_stride_block, a.v_stride_token, a.v_stride_head = v_cache.stride()[:3]
    a.bt_stride = bt.stride(0)
    a.num_seqs, a.num_q_heads, a.head_dim = n, hq, d
    a.num_kv_heads, a.block_size = k_cache.shape[2], k_cache.shape[1]
    a.dtype = _dtype_code(q)
    a.num_threads = num_threads
    a.scale = float(scale)
    rc = oracle_lib().dk_oracle_paged_attention(ctypes.byref(a))
    if rc != 0:
        raise RuntimeError(f"dk_oracle_paged_attention failed ({rc})")
    if info is not None:
        info["threads_used"], info["units"] = int(a.threads_used), int(a.units)
    return out


def max_threads() -> int:
    return int(oracle_lib().dk_oracle_max_threads())


def reference_kernel(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, workspace=None,
                     stream=None) -> None:
    """Run the reference's kernels (built from its source) on device tensors."""
    import torch

    a = DkRefArgs()
    a.out, a.q = out.data_ptr(), q.data_ptr()
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.block_tables, a.seq_lens = block_tables.data_ptr(), seq_lens.data_ptr()
    a.max_partitions = 1
    if workspace is not None and workspace[0].numel() > 0:
        a.tmp_out, a.max_logits, a.exp_sums = (t.data_ptr() for t in workspace)
        a.max_partitions = workspace[0].shape[2]
    a.q_stride_seq, a.q_stride_head = q.stride(0), q.stride(1)
    a.out_stride_seq, a.out_stride_head = out.stride(0), out.stride(1)
    a.k_stride_block, a.k_stride_token, a.k_stride_head = k_cache.stride()[:3]
    a.v_stride_block, a.v_stride_token, a.v_stride_head = v_cache.stride()[:3]
    a.bt_stride = block_tables.stride(0)
    a.num_seqs, a.num_q_heads, a.head_dim = q.shape
    a.num_kv_heads, a.block_size = k_cache.shape[2], k_cache.shape[1]
    a.max_seq_len = int(max_seq_len)
    a.dtype = _dtype_code(q)
    a.scale = float(scale)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = ref_lib().dk_ref_paged_attention_decode(ctypes.byref(a), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"reference kernel launch failed ({rc})")


def reference_workspace(num_seqs, num_q_heads, head_dim, max_seq_len, device):
    """The reference's own workspace sizing (decode_kernels/ops.py:71-80)."""
    import math

    import torch

    if max_seq_len <= 512:
        e = torch.empty(0, dtype=torch.float32, device=device)
        return e, e, e
    parts = max(1, math.ceil(max_seq_len / 512))
    tmp = torch.empty(num_seqs, num_q_heads, parts, head_dim, dtype=torch.float32, device=device)
    ml = torch.empty(num_seqs, num_q_heads, parts, dtype=torch.float32, device=device)
    return tmp, ml, torch.empty_like(ml)


def cpu_count() -> int:
    return os.cpu_count() or 1
