"""decodekernels_b200: paged-attention decode for NVIDIA B200 (sm_100a).

A from-scratch, B200-native implementation of DecodeKernels'
``paged_attention_decode`` path behind the same torch op and Python API:

    import decodekernels_b200 as dk
    out = dk.paged_attention_decode(q, k_cache, v_cache, block_tables, seq_lens)
    dk.reshape_and_cache(key, value, k_cache, v_cache, slot_mapping)   # the paged-KV write before it

The kernels live in ``libdk_b200.so`` (C ABI: ``include/dk_paged_attention.h``);
``torch.ops.decode_kernels.paged_attention_decode`` is registered by
``libdk_b200_torch.so``.  Build both with ``python -m decodekernels_b200.build``.
"""

from .ops import (
    FLAG_PERSISTENT,
    MAX_GQA_GROUP,
    PARTITION_SIZE,
    SUPPORTED_HEAD_DIMS,
    alloc_workspace,
    is_available,
    merge_lse,
    num_partitions,
    paged_attention_decode,
    paged_attention_decode_lse,
    reshape_and_cache,
)

__all__ = [
    "FLAG_PERSISTENT",
    "MAX_GQA_GROUP",
    "PARTITION_SIZE",
    "SUPPORTED_HEAD_DIMS",
    "alloc_workspace",
    "is_available",
    "merge_lse",
    "num_partitions",
    "paged_attention_decode",
    "paged_attention_decode_lse",
    "reshape_and_cache",
]
__version__ = "0.8.0"
