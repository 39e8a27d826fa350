"""``decode_kernels.vllm_plugin:register``, the object DecodeKernels names in
its ``vllm.general_plugins`` entry point (``pyproject.toml:22-23``); here it is
decodekernels_b200's plugin (a no-op unless ``DECODE_KERNELS_VLLM=1``)."""

from decodekernels_b200.vllm_plugin import register

__all__ = ["register"]
