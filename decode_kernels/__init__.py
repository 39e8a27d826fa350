"""``decode_kernels``: DecodeKernels' import path, served by decodekernels_b200.

Callers written against DecodeKernels keep their imports::

    import decode_kernels as dk
    out = dk.paged_attention_decode(q, k_cache, v_cache, block_tables, seq_lens)
    ws = dk.alloc_workspace(num_seqs, num_q_heads, head_dim, max_seq_len, "cuda")

and get this library's sm_100a kernels behind the same names, signatures,
defaults and errors (DecodeKernels ``decode_kernels/__init__.py:1-27``,
``decode_kernels/ops.py:14-116``); importing it registers
``torch.ops.decode_kernels.paged_attention_decode`` with the reference's
schema.  Only the attention path is provided: the reference's ``gemm``,
``rms_norm``, ``fused_add_rms_norm`` and ``silu_and_mul`` are not part of
this library.  Install either this package or the reference, not both: both
register the ``decode_kernels`` torch op namespace.
"""

from decodekernels_b200 import __version__
from decodekernels_b200.ops import PARTITION_SIZE, alloc_workspace, is_available, paged_attention_decode

from . import ops  # noqa: F401  (decode_kernels.ops, as in the reference)

__all__ = ["PARTITION_SIZE", "alloc_workspace", "is_available", "paged_attention_decode"]
