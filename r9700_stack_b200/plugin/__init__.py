"""vLLM-facing entry points.

``register()`` (group ``vllm.general_plugins``) runs in every vLLM process and registers, each behind
an ``R9K_DISABLE`` opt-out:

* ``ops``    -- fake (meta) implementations of every ``torch.ops.r9k`` op, so graphs that call them
               trace under ``torch.compile`` and capture into CUDA graphs;
* ``quant``  -- quantization config ``compressed-tensors`` (overrides vLLM's: NVFP4 and fp8 linears
               run on this library's tcgen05 GEMMs, ``plugin.quant_ct``) and ``exl3`` (trellis
               linears, ``plugin.quant_exl3``);
* ``models`` -- model classes for the BASELINE architectures (``plugin.models.ARCHS``): vLLM's own
               classes with this library's fused RMSNorm installed;
* ``attn``   -- attention backend ``CUSTOM``: paged fp8 KV attention on this library's kernels
               (``plugin.attention``).

``plugin.platform.detect()`` (group ``vllm.platform_plugins``) selects the B200 platform class, whose
device communicator routes tensor-parallel all-reduces through this framework's NVLink collectives.
``R9K_PLATFORM=0`` keeps vLLM's own platform. The serving path where every named hot op is this
library's is its own engine (``engine``, ``serve``); the vLLM surface lets vLLM users run its kernels.
Reference: r9700_vllm/__init__.py:27-85 (register), r9700_vllm/platform.py:15-40 (detect).
"""
from __future__ import annotations

import logging

from .. import knobs

log = logging.getLogger("vllm.r9700_stack_b200")
_registered: list[str] | None = None


def register() -> list[str]:
    """Register everything not opted out; returns what was registered (idempotent)."""
    global _registered
    if _registered is not None:
        return _registered
    done: list[str] = []
    if knobs.disabled("plugin"):
        _registered = done
        return done
    if not knobs.disabled("ops"):
        from .fake_ops import register_fakes

        done.append(f"ops:{register_fakes()}")
    if not knobs.disabled("quant"):
        from . import quant_ct, quant_exl3  # noqa: F401  (the decorators register the configs)

        done.append("quant:compressed-tensors,exl3")
    if not knobs.disabled("models"):
        from vllm import ModelRegistry

        from .models import ARCHS

        for arch, qual in ARCHS.items():
            ModelRegistry.register_model(arch, qual)
        done.append("models:" + ",".join(ARCHS))
    if not knobs.disabled("attn"):
        from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

        register_backend(AttentionBackendEnum.CUSTOM, "r9700_stack_b200.plugin.attention.R9kAttentionBackend")
        done.append("attn:CUSTOM")
    _registered = done
    log.info("r9700_stack_b200 registered: %s", ", ".join(done) or "nothing")
    return done
