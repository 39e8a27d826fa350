"""vLLM general-plugin entry point (``vllm.general_plugins``).

vLLM imports this in every process it starts (API server, engine core,
workers).  It is a no-op unless ``DECODE_KERNELS_VLLM=1``, so installing the
package never changes vLLM's behaviour by itself (the reference's switches,
``decode_kernels/vllm_plugin.py:14-20``):

    DECODE_KERNELS_VLLM=1             enable
    DECODE_KERNELS_OPS=attention      which ops to swap (default: attention)
"""

import os


def register() -> None:
    if os.environ.get("DECODE_KERNELS_VLLM", "0") != "1":
        return
    from .vllm_patch import apply

    ops = os.environ.get("DECODE_KERNELS_OPS", "attention")
    apply([o.strip() for o in ops.split(",") if o.strip()])
