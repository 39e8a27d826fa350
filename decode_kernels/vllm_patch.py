"""``decode_kernels.vllm_patch``: decodekernels_b200's patch of vLLM's attention
forward (``apply``, ``stats``, ``reset_stats``), under the reference's module
name (DecodeKernels ``decode_kernels/vllm_patch.py``)."""

from decodekernels_b200.vllm_patch import apply, reset_stats, stats

__all__ = ["apply", "reset_stats", "stats"]
