"""``decode_kernels.ops`` for the attention path: the reference's constants and
wrapper functions (DecodeKernels ``decode_kernels/ops.py:14-116``), which
decodekernels_b200 implements."""

from decodekernels_b200.ops import (
    MAX_GQA_GROUP,
    PARTITION_SIZE,
    SUPPORTED_HEAD_DIMS,
    alloc_workspace,
    is_available,
    num_partitions,
    paged_attention_decode,
)

__all__ = ["MAX_GQA_GROUP", "PARTITION_SIZE", "SUPPORTED_HEAD_DIMS", "alloc_workspace", "is_available",
           "num_partitions", "paged_attention_decode"]
