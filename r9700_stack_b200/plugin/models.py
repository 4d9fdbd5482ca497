"""vLLM model classes for the architectures of the BASELINE configurations, with this library's
kernels installed into vLLM's own layer modules.

Each class subclasses vLLM's stock implementation of the architecture (so vLLM's loader, scheduler and
KV-cache manager work unchanged) and, after construction, ``install()`` rebinds the forward of every
RMSNorm module (plain and Gemma-style ``x * (1 + w)``) to ``rmsnorm_quant``, the fused residual add +
RMSNorm kernel. Linear layers reach this library through the quantization configs of this package
(``quant_ct``, ``quant_exl3``) and attention through the ``CUSTOM`` backend (``attention``); the
engine of this repository (``engine``) remains the path where every hot op is this library's.
Reference: r9700_vllm/__init__.py:40-48 (ModelRegistry.register_model of the ARCHS dicts),
r9700_vllm/models/qwen4_exp.py:196-208 (construct, then install per instance).
"""
from __future__ import annotations

import types

import torch

from .. import _native

# vLLM architecture name -> "module:class" of this package
ARCHS = {
    "Qwen3NextForCausalLM": "r9700_stack_b200.plugin.models:R9kQwen3NextForCausalLM",
    "Qwen3_5ForCausalLM": "r9700_stack_b200.plugin.models:R9kQwen3_5ForCausalLM",
    "Qwen3_5MoeForCausalLM": "r9700_stack_b200.plugin.models:R9kQwen3_5MoeForCausalLM",
    "Glm4MoeForCausalLM": "r9700_stack_b200.plugin.models:R9kGlm4MoeForCausalLM",
    "DeepseekV3ForCausalLM": "r9700_stack_b200.plugin.models:R9kDeepseekV3ForCausalLM",
}


def rmsnorm_forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
    """vLLM RMSNorm semantics (residual is added first and returned as the new residual) on the fused
    kernel; shapes the kernel does not take (not 2-D bf16, width not a multiple of 32) keep vLLM's."""
    if x.dtype != torch.bfloat16 or x.shape[-1] % 32 != 0 or (residual is not None and residual.dtype != x.dtype):
        return self._r9k_stock_forward(x, residual)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    y = torch.empty_like(x2)
    new_res = torch.empty_like(x2) if residual is not None else None
    _native.ops().rmsnorm_quant(x2, residual.reshape(-1, shape[-1]).contiguous() if residual is not None else None,
                                new_res, self.weight.data.to(torch.bfloat16), float(self.variance_epsilon),
                                bool(self._r9k_plus_one), y, None, None)
    if residual is None:
        return y.view(shape)
    return y.view(shape), new_res.view(shape)


def install(model: torch.nn.Module) -> int:
    """Rebind every RMSNorm / GemmaRMSNorm module of ``model`` to the fused kernel. Returns the count."""
    from vllm.model_executor.layers.layernorm import GemmaRMSNorm, RMSNorm

    n = 0
    for mod in model.modules():
        if isinstance(mod, (RMSNorm, GemmaRMSNorm)) and not hasattr(mod, "_r9k_stock_forward"):
            if getattr(mod, "has_weight", True) is False:
                continue
            mod._r9k_plus_one = isinstance(mod, GemmaRMSNorm)
            mod._r9k_stock_forward = mod.forward
            mod.forward = types.MethodType(rmsnorm_forward, mod)
            n += 1
    return n


def _make(base_path: str, name: str):
    import importlib

    mod, cls = base_path.split(":")
    base = getattr(importlib.import_module(mod), cls)

    def __init__(self, *args, **kwargs):
        base.__init__(self, *args, **kwargs)
        self.r9k_installed = install(self)

    return type(name, (base,), {"__init__": __init__, "__module__": __name__})


_BASES = {
    "R9kQwen3NextForCausalLM": "vllm.model_executor.models.qwen3_next:Qwen3NextForCausalLM",
    "R9kQwen3_5ForCausalLM": "vllm.model_executor.models.qwen3_5:Qwen3_5ForCausalLM",
    "R9kQwen3_5MoeForCausalLM": "vllm.model_executor.models.qwen3_5:Qwen3_5MoeForCausalLM",
    "R9kGlm4MoeForCausalLM": "vllm.model_executor.models.glm4_moe:Glm4MoeForCausalLM",
    "R9kDeepseekV3ForCausalLM": "vllm.model_executor.models.deepseek_v2:DeepseekV3ForCausalLM",
}


def __getattr__(name):
    # classes are built on first use: importing vLLM's model modules pulls in its CUDA layers
    if name in _BASES:
        cls = _make(_BASES[name], name)
        globals()[name] = cls
        return cls
    raise AttributeError(name)
