"""ctypes bindings of the C ABI (``include/dk_paged_attention.h``).

This is the torch-free boundary: every call passes raw device pointers and
element strides to ``libdk_b200.so``.  The helpers here take torch tensors
only to read their pointers, shapes and strides; tests use them to drive the
C ABI directly (including options the torch op does not expose: a fixed
partition size, the CUDA-core path).

The library is loaded from ``decodekernels_b200/lib/``; if it is missing,
``load()`` raises -- there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libdk_b200.so"

DK_DTYPE_FLOAT16 = 0
DK_DTYPE_BFLOAT16 = 1
DK_DTYPE_FP8_E4M3 = 2
DK_PATH_NONE, DK_PATH_TMA_MMA, DK_PATH_SIMT = 0, 1, 2
DK_FLAG_FORCE_SIMT = 1
DK_FLAG_FORCE_FUSED_MERGE = 2
DK_FLAG_PERSISTENT = 4
DK_MAX_GQA_GROUP = 8
DK_TILE_TOKENS = 64
DK_REF_PARTITION_SIZE = 512

DK_NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024

EXPORTED = ("dk_paged_attention_decode", "dk_plan", "dk_num_partitions", "dk_last_error",
            "dk_device_wait_timeouts", "dk_version", "dk_paged_attention_decode_noalloc", "dk_reshape_and_cache",
            "dk_paged_attention_decode_lse", "dk_merge_lse", "dk_exchange_merge_lse", "dk_gather_heads",
            "dk_paged_attention_decode_gather")


class DkPagedAttnArgs(ctypes.Structure):
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
        ("merge_counters", ctypes.c_void_p),
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
        ("num_blocks", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32),
        ("max_partitions", ctypes.c_int32),
        ("partition_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("kv_fp8", ctypes.c_int32),
        ("k_scale", ctypes.c_float),
        ("v_scale", ctypes.c_float),
    ]


class DkCacheWriteArgs(ctypes.Structure):
    _fields_ = [
        ("key", ctypes.c_void_p),
        ("value", ctypes.c_void_p),
        ("key_cache", ctypes.c_void_p),
        ("value_cache", ctypes.c_void_p),
        ("slot_mapping", ctypes.c_void_p),
        ("key_stride_token", ctypes.c_int64),
        ("key_stride_head", ctypes.c_int64),
        ("value_stride_token", ctypes.c_int64),
        ("value_stride_head", ctypes.c_int64),
        ("k_stride_block", ctypes.c_int64),
        ("k_stride_token", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("v_stride_block", ctypes.c_int64),
        ("v_stride_token", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("num_tokens", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("cache_dtype", ctypes.c_int32),
        ("k_scale", ctypes.c_float),
        ("v_scale", ctypes.c_float),
    ]


class DkLseMergeArgs(ctypes.Structure):
    _fields_ = [
        ("parts", ctypes.c_void_p),
        ("part_stride", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("out_stride_seq", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("num_parts", ctypes.c_int32),
        ("num_seqs", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("out_partial", ctypes.c_int32),
    ]


DK_MAX_PEERS = 8


class DkPeerExchangeArgs(ctypes.Structure):
    _fields_ = [
        ("partial", ctypes.c_void_p),
        ("recv", ctypes.c_void_p * DK_MAX_PEERS),
        ("flags", ctypes.c_void_p * DK_MAX_PEERS),
        ("state", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_stride_seq", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("num_seqs", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("wait_limit_ms", ctypes.c_uint32),
    ]


class DkPeerGatherArgs(ctypes.Structure):
    _fields_ = [
        ("local", ctypes.c_void_p),
        ("local_stride_seq", ctypes.c_int64),
        ("local_stride_head", ctypes.c_int64),
        ("recv", ctypes.c_void_p * DK_MAX_PEERS),
        ("flags", ctypes.c_void_p * DK_MAX_PEERS),
        ("state", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_stride_seq", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("num_seqs", ctypes.c_int32),
        ("heads_per_rank", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("wait_limit_ms", ctypes.c_uint32),
    ]


class DkPlan(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_int32),
        ("partition_size", ctypes.c_int32),
        ("num_partitions", ctypes.c_int32),
        ("split", ctypes.c_int32),
        ("num_ctas", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("launches", ctypes.c_int32),
        ("ctas_per_sm", ctypes.c_int32),
        ("fit_min_partition", ctypes.c_int32),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libdk_b200.so (once) and declare the exported signatures."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run `python -m decodekernels_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.dk_paged_attention_decode.argtypes = [ctypes.POINTER(DkPagedAttnArgs), ctypes.c_void_p]
        lib.dk_paged_attention_decode.restype = ctypes.c_int
        lib.dk_paged_attention_decode_noalloc.argtypes = [ctypes.POINTER(DkPagedAttnArgs), ctypes.c_void_p]
        lib.dk_paged_attention_decode_noalloc.restype = ctypes.c_int
        lib.dk_plan.argtypes = [ctypes.POINTER(DkPagedAttnArgs), ctypes.POINTER(DkPlan)]
        lib.dk_plan.restype = ctypes.c_int
        lib.dk_num_partitions.argtypes = [ctypes.c_int32] * 6
        lib.dk_num_partitions.restype = ctypes.c_int32
        lib.dk_last_error.argtypes = []
        lib.dk_last_error.restype = ctypes.c_char_p
        lib.dk_device_wait_timeouts.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_uint32)]
        lib.dk_device_wait_timeouts.restype = ctypes.c_int
        lib.dk_version.argtypes = []
        lib.dk_version.restype = ctypes.c_int32
        lib.dk_reshape_and_cache.argtypes = [ctypes.POINTER(DkCacheWriteArgs), ctypes.c_void_p]
        lib.dk_reshape_and_cache.restype = ctypes.c_int
        lib.dk_paged_attention_decode_lse.argtypes = [ctypes.POINTER(DkPagedAttnArgs), ctypes.c_void_p,
                                                      ctypes.c_void_p]
        lib.dk_paged_attention_decode_lse.restype = ctypes.c_int
        lib.dk_merge_lse.argtypes = [ctypes.POINTER(DkLseMergeArgs), ctypes.c_void_p]
        lib.dk_merge_lse.restype = ctypes.c_int
        lib.dk_exchange_merge_lse.argtypes = [ctypes.POINTER(DkPeerExchangeArgs), ctypes.c_void_p]
        lib.dk_exchange_merge_lse.restype = ctypes.c_int
        lib.dk_gather_heads.argtypes = [ctypes.POINTER(DkPeerGatherArgs), ctypes.c_void_p]
        lib.dk_gather_heads.restype = ctypes.c_int
        lib.dk_paged_attention_decode_gather.argtypes = [ctypes.POINTER(DkPagedAttnArgs),
                                                         ctypes.POINTER(DkPeerGatherArgs), ctypes.c_void_p]
        lib.dk_paged_attention_decode_gather.restype = ctypes.c_int
        _lib = lib
        return lib


def last_error() -> str:
    return load().dk_last_error().decode()


def version() -> int:
    return int(load().dk_version())


def num_partitions(num_seqs: int, num_kv_heads: int, head_dim: int, block_size: int, max_seq_len: int,
                   device: int = -1) -> int:
    n = load().dk_num_partitions(num_seqs, num_kv_heads, head_dim, block_size, max_seq_len, device)
    if n < 0:
        raise ValueError(f"dk_num_partitions rejected ({num_seqs}, {num_kv_heads}, {head_dim}, {max_seq_len})")
    return int(n)


def wait_timeouts(device: int = 0) -> int:
    count = ctypes.c_uint32(0)
    rc = load().dk_device_wait_timeouts(device, ctypes.byref(count))
    if rc != 0:
        raise RuntimeError(f"dk_device_wait_timeouts failed ({rc}): {last_error()}")
    return int(count.value)


def _dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float16:
        return DK_DTYPE_FLOAT16
    if t.dtype == torch.bfloat16:
        return DK_DTYPE_BFLOAT16
    return -1


def make_args(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, workspace=None,
              partition_size: int = 0, force_simt: bool = False, flags: int = 0, k_scale: float = 1.0,
              v_scale: float = 1.0) -> DkPagedAttnArgs:
    """Fill the C struct from tensors (pointers + element strides).  A uint8 /
    float8_e4m3fn cache is read as e4m3 with the per-tensor scales."""
    a = DkPagedAttnArgs()
    a.out = out.data_ptr()
    a.q = q.data_ptr()
    a.k_cache = k_cache.data_ptr()
    a.v_cache = v_cache.data_ptr()
    a.block_tables = block_tables.data_ptr()
    a.seq_lens = seq_lens.data_ptr()
    if workspace is not None and workspace[0].numel() > 0:
        tmp_out, max_logits, exp_sums = workspace[:3]
        a.tmp_out, a.max_logits, a.exp_sums = tmp_out.data_ptr(), max_logits.data_ptr(), exp_sums.data_ptr()
        a.max_partitions = tmp_out.shape[2]
        if len(workspace) > 3 and workspace[3] is not None and workspace[3].numel() > 0:
            a.merge_counters = workspace[3].data_ptr()  # single-launch merge
    a.q_stride_seq, a.q_stride_head = q.stride(0), q.stride(1)
    a.out_stride_seq, a.out_stride_head = out.stride(0), out.stride(1)
    a.k_stride_block, a.k_stride_token, a.k_stride_head = k_cache.stride()[:3]
    a.v_stride_block, a.v_stride_token, a.v_stride_head = v_cache.stride()[:3]
    a.bt_stride = block_tables.stride(0)
    a.num_seqs, a.num_q_heads, a.head_dim = q.shape
    a.num_kv_heads = k_cache.shape[2]
    a.block_size = k_cache.shape[1]
    a.num_blocks = k_cache.shape[0]
    a.max_seq_len = int(max_seq_len)
    a.partition_size = int(partition_size)
    a.dtype = _dtype_code(q)
    a.flags = (DK_FLAG_FORCE_SIMT if force_simt else 0) | flags
    a.scale = float(scale)
    a.kv_fp8 = 1 if _cache_dtype_code(k_cache) == DK_DTYPE_FP8_E4M3 else 0
    a.k_scale, a.v_scale = float(k_scale), float(v_scale)
    return a


def plan(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, workspace=None,
         partition_size: int = 0, force_simt: bool = False, flags: int = 0, k_scale: float = 1.0,
         v_scale: float = 1.0) -> dict:
    a = make_args(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, workspace, partition_size,
                  force_simt, flags, k_scale, v_scale)
    p = DkPlan()
    rc = load().dk_plan(ctypes.byref(a), ctypes.byref(p))
    if rc != 0:
        raise RuntimeError(f"dk_plan failed ({rc}): {last_error()}")
    return p.as_dict()


def decode(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, workspace=None,
           partition_size: int = 0, force_simt: bool = False, stream=None, flags: int = 0, k_scale: float = 1.0,
           v_scale: float = 1.0) -> int:
    """dk_paged_attention_decode on ``stream`` (default: torch's current stream).

    Returns 0; raises RuntimeError with the library's message otherwise."""
    import torch

    a = make_args(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, workspace, partition_size,
                  force_simt, flags, k_scale, v_scale)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream if q.is_cuda else 0
    rc = load().dk_paged_attention_decode(ctypes.byref(a), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_paged_attention_decode failed ({rc}): {last_error()}")
    return rc


def decode_noalloc(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, stream=None,
                   flags: int = 0, k_scale: float = 1.0, v_scale: float = 1.0) -> int:
    """dk_paged_attention_decode_noalloc: the decode for callers that cannot
    allocate device memory (plugin hosts and runtimes that own all memory
    besides a kernel's inputs and outputs, FFI hosts without a CUDA
    allocator).  Split-K partials go to the library's static scratch of
    DK_NOALLOC_SCRATCH_BYTES; calls that would need more are rejected
    (RuntimeError).  Calls that overlap on the GPU share that scratch and race.
    """
    import torch

    a = make_args(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, None, 0, False, flags,
                  k_scale, v_scale)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream if q.is_cuda else 0
    rc = load().dk_paged_attention_decode_noalloc(ctypes.byref(a), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_paged_attention_decode_noalloc failed ({rc}): {last_error()}")
    return rc


def _cache_dtype_code(t) -> int:
    import torch

    if t.dtype in (torch.uint8, torch.float8_e4m3fn):
        return DK_DTYPE_FP8_E4M3
    return _dtype_code(t)


def make_cache_write_args(key, value, key_cache, value_cache, slot_mapping, k_scale: float = 1.0,
                          v_scale: float = 1.0) -> DkCacheWriteArgs:
    """Fill the paged-KV write struct from tensors (pointers + element strides)."""
    a = DkCacheWriteArgs()
    a.key, a.value = key.data_ptr(), value.data_ptr()
    a.key_cache, a.value_cache = key_cache.data_ptr(), value_cache.data_ptr()
    a.slot_mapping = slot_mapping.data_ptr()
    a.key_stride_token, a.key_stride_head = key.stride(0), key.stride(1)
    a.value_stride_token, a.value_stride_head = value.stride(0), value.stride(1)
    a.k_stride_block, a.k_stride_token, a.k_stride_head = key_cache.stride()[:3]
    a.v_stride_block, a.v_stride_token, a.v_stride_head = value_cache.stride()[:3]
    a.num_tokens, a.num_kv_heads, a.head_dim = key.shape
    a.num_blocks, a.block_size = key_cache.shape[0], key_cache.shape[1]
    a.dtype = _dtype_code(key)
    a.cache_dtype = _cache_dtype_code(key_cache)
    a.k_scale, a.v_scale = float(k_scale), float(v_scale)
    return a


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, k_scale: float = 1.0, v_scale: float = 1.0,
                      stream=None) -> int:
    """dk_reshape_and_cache on ``stream`` (default: torch's current stream)."""
    import torch

    a = make_cache_write_args(key, value, key_cache, value_cache, slot_mapping, k_scale, v_scale)
    if stream is None:
        stream = torch.cuda.current_stream(key.device).cuda_stream if key.is_cuda else 0
    rc = load().dk_reshape_and_cache(ctypes.byref(a), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_reshape_and_cache failed ({rc}): {last_error()}")
    return rc


def decode_lse(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, partial, workspace=None,
               partition_size: int = 0, stream=None, flags: int = 0, k_scale: float = 1.0,
               v_scale: float = 1.0) -> int:
    """dk_paged_attention_decode_lse: fp32 rows (o, lse, pad) into ``partial`` [n, Hq, D + 4]."""
    import torch

    a = make_args(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, partial, workspace, partition_size,
                  False, flags, k_scale, v_scale)
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream if q.is_cuda else 0
    rc = load().dk_paged_attention_decode_lse(ctypes.byref(a), ctypes.c_void_p(partial.data_ptr()),
                                              ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_paged_attention_decode_lse failed ({rc}): {last_error()}")
    return rc


def make_lse_merge_args(parts, out) -> DkLseMergeArgs:
    """Struct for parts [R, n, Hq, D + 4] fp32 and out [n, Hq, D] (fp16 / bf16) or [n, Hq, D + 4] fp32."""
    import torch

    a = DkLseMergeArgs()
    a.parts, a.part_stride = parts.data_ptr(), parts.stride(0)
    a.out, a.out_stride_seq, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.num_parts, a.num_seqs, a.num_q_heads = parts.shape[0], parts.shape[1], parts.shape[2]
    a.head_dim = parts.shape[3] - 4
    a.out_partial = 1 if out.dtype == torch.float32 else 0
    a.dtype = _dtype_code(out) if not a.out_partial else DK_DTYPE_FLOAT16
    return a


def merge_lse(parts, out, stream=None) -> int:
    """dk_merge_lse on ``stream`` (default: torch's current stream)."""
    import torch

    a = make_lse_merge_args(parts, out)
    if stream is None:
        stream = torch.cuda.current_stream(parts.device).cuda_stream if parts.is_cuda else 0
    rc = load().dk_merge_lse(ctypes.byref(a), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_merge_lse failed ({rc}): {last_error()}")
    return rc


def gather_heads(local, recv_ptrs, flag_ptrs, state, out, rank: int, world: int, wait_limit_ms: int = 0,
                 stream=None) -> int:
    """dk_gather_heads: push ``local`` [n, Hq / world, D] (this rank's heads)
    to every GPU's receive buffer, wait for every rank's flag, copy all heads
    into ``out`` [n, Hq, D]."""
    import torch

    a = DkPeerGatherArgs()
    a.local, a.local_stride_seq, a.local_stride_head = local.data_ptr(), local.stride(0), local.stride(1)
    for r in range(world):
        a.recv[r] = recv_ptrs[r]
        a.flags[r] = flag_ptrs[r]
    a.state = state.data_ptr()
    a.out, a.out_stride_seq, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.rank, a.world = rank, world
    a.num_seqs, a.heads_per_rank, a.head_dim = local.shape[0], local.shape[1], local.shape[2]
    a.dtype = _dtype_code(out)
    a.wait_limit_ms = wait_limit_ms
    if stream is None:
        stream = torch.cuda.current_stream(local.device).cuda_stream
    rc = load().dk_gather_heads(ctypes.byref(a), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_gather_heads failed ({rc}): {last_error()}")
    return rc


def decode_gather(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, workspace, recv_ptrs, flag_ptrs,
                  state, out, rank: int, world: int, wait_limit_ms: int = 0, flags: int = 0, k_scale: float = 1.0,
                  v_scale: float = 1.0, stream=None) -> int:
    """dk_paged_attention_decode_gather: decode this rank's heads ``q``
    [n, Hq / world, D] with the output rows stored straight into every
    rank's receive slot, then all heads into ``out`` [n, Hq, D]."""
    import torch

    a = make_args(q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, out, workspace, 0, False, flags,
                  k_scale, v_scale)
    g = DkPeerGatherArgs()
    g.local = 0
    for r in range(world):
        g.recv[r] = recv_ptrs[r]
        g.flags[r] = flag_ptrs[r]
    g.state = state.data_ptr()
    g.out, g.out_stride_seq, g.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    g.rank, g.world = rank, world
    g.num_seqs, g.heads_per_rank, g.head_dim = q.shape[0], q.shape[1], q.shape[2]
    g.dtype = _dtype_code(out)
    g.wait_limit_ms = wait_limit_ms
    if stream is None:
        stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = load().dk_paged_attention_decode_gather(ctypes.byref(a), ctypes.byref(g), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_paged_attention_decode_gather failed ({rc}): {last_error()}")
    return rc


def exchange_merge_lse(partial, recv_ptrs, flag_ptrs, state, out, rank: int, world: int, wait_limit_ms: int = 0,
                       stream=None) -> int:
    """dk_exchange_merge_lse: push ``partial`` [n, Hq, D + 4] to every GPU's
    receive buffer, wait for every rank's flag, merge into ``out`` [n, Hq, D]."""
    import torch

    a = DkPeerExchangeArgs()
    a.partial = partial.data_ptr()
    for r in range(world):
        a.recv[r] = recv_ptrs[r]
        a.flags[r] = flag_ptrs[r]
    a.state = state.data_ptr()
    a.out, a.out_stride_seq, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.rank, a.world = rank, world
    a.num_seqs, a.num_q_heads, a.head_dim = partial.shape[0], partial.shape[1], partial.shape[2] - 4
    a.dtype = _dtype_code(out)
    a.wait_limit_ms = wait_limit_ms
    if stream is None:
        stream = torch.cuda.current_stream(partial.device).cuda_stream
    rc = load().dk_exchange_merge_lse(ctypes.byref(a), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"dk_exchange_merge_lse failed ({rc}): {last_error()}")
    return rc
