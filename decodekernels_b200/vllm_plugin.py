"""Entry point that vLLM calls through its ``vllm.general_plugins`` group.

vLLM runs every registered general plugin in each of its processes, so this
function must stay cheap and must not change anything on its own: it returns
at once unless the environment variable ``DECODE_KERNELS_VLLM`` is ``1``.
When it is, the attention forward of vLLM's FlashAttention backend is
patched (``vllm_patch.apply``) for the op names listed, comma-separated, in
``DECODE_KERNELS_OPS`` (default ``attention``, the only op this library
implements; other names are logged and skipped).  The variable names and
their meaning are DecodeKernels' (``decode_kernels/vllm_plugin.py:14-20``).
"""

import os


def register() -> None:
    if os.environ.get("DECODE_KERNELS_VLLM", "0") != "1":
        return
    from .vllm_patch import apply

    ops = os.environ.get("DECODE_KERNELS_OPS", "attention")
    apply([o.strip() for o in ops.split(",") if o.strip()])
