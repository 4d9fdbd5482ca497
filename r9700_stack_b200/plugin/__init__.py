"""vLLM-facing entry points.

``register()`` (group ``vllm.general_plugins``) loads the kernel library and registers fake (meta)
implementations of every ``torch.ops.r9k`` op, so graphs that call them can be traced by
``torch.compile``; ``plugin.platform.detect()`` (group ``vllm.platform_plugins``) selects the B200
platform class, whose device communicator routes tensor-parallel all-reduces through this
framework's NVLink collectives (``parallel.collectives``) and everything else through NCCL. The
model execution path of this framework is its own engine (``engine``, ``serve``): the named hot paths
here must not fall back to library kernels, which vLLM's CUDA model runner would call.
``R9K_DISABLE=plugin`` turns the registration off; ``R9K_PLATFORM=0`` keeps vLLM's own platform.
Reference: r9700_vllm/__init__.py:27-85 (register), r9700_vllm/platform.py:15-40 (detect).
"""
from __future__ import annotations

import logging

from .. import knobs

log = logging.getLogger("vllm.r9700_stack_b200")
_registered = False


def register() -> None:
    global _registered
    if _registered or knobs.disabled("plugin"):
        return
    from .fake_ops import register_fakes

    n = register_fakes()
    _registered = True
    log.info("r9700_stack_b200: %d kernel ops registered (fake impls for tracing)", n)
