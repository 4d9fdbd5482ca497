"""vLLM quantization config "compressed-tensors", served by this library's tcgen05 GEMMs.

Registered under vLLM's own name, so it replaces the stock config for every compressed-tensors
checkpoint (vLLM warns once that the name is overwritten). The stock config still parses the
checkpoint's quantization groups and builds each layer's parameters under the checkpoint's tensor
names; per layer, schemes this library serves get their class swapped (that instance only) for a
subclass whose load-time transform and forward call ``torch.ops.r9k``:

* NVFP4 (``CompressedTensorsW4A4Fp4`` / ``CompressedTensorsW4A16Fp4``: e2m1 weights, e4m3 scale per 16,
  fp32 global scale): converted to MXFP4 at load (MSE search over +-2 exponent shifts per 32-block,
  the same conversion as the engine's loader) and run as MXFP4 x MXFP8 on
  ``tcgen05.mma kind::mxf8f6f4.block_scale``. Shards of a fused layer (qkv, gate/up) carry their own
  global scales; each shard converts with its own.
* fp8 weights (``CompressedTensorsW8A8Fp8``: per-channel or 128x128 block scales): requantised to
  MXFP8 at load (the fp8 bytes are exact in the dequantised fp32 tensor) and run on the same GEMM.

Anything else keeps the stock scheme. ``R9K_DISABLE=quant`` keeps the stock config entirely.
Reference: r9700_vllm/quant/ct.py:347-462 (the same override, on RDNA4 kernels),
r9700_vllm/quant/nvfp4.py:78-112 (load-time NVFP4 -> MXFP4).
"""
from __future__ import annotations

import torch
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.compressed_tensors.compressed_tensors import CompressedTensorsConfig
from vllm.model_executor.layers.quantization.compressed_tensors.schemes import (
    CompressedTensorsW4A4Fp4,
    CompressedTensorsW4A16Fp4,
    CompressedTensorsW8A8Fp8,
)

from .. import knobs
from ..ops import linear as L


def _tiled() -> bool:
    return knobs.get("R9K_WEIGHT_TILED") != "0"


def mx_apply(w: L.MXWeight, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """y = x @ W^T (+ bias) for any leading shape of x: MXFP8 activations, tcgen05 GEMM, bf16 result."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    y = L.mx_linear(L.quant_act(x2.contiguous()), w)
    if bias is not None:
        y = y + bias
    return y.reshape(*lead, w.N)


def nvfp4_to_mx(packed: torch.Tensor, s16: torch.Tensor, gscale: torch.Tensor, widths: list[int]) -> L.MXWeight:
    """Checkpoint NVFP4 rows (packed e2m1 [N, K/2], e4m3 scales [N, K/16], one global scale per shard of
    ``widths`` rows) -> one MXFP4 weight. Rows of a shard are converted with that shard's scale."""
    g = gscale.float().reshape(-1)
    s16b = s16.contiguous().view(torch.uint8)
    if g.numel() <= 1 or bool((g == g[0]).all()):
        return L.mx_from_nvfp4(packed.contiguous(), s16b, float(g[0]), search=True)
    parts, r0 = [], 0
    for i, n in enumerate(widths):
        part = L.mx_from_nvfp4(packed[r0:r0 + n].contiguous(), s16b[r0:r0 + n].contiguous(), float(g[i]), search=True)
        parts.append(part.dequant())
        r0 += n
    # MX block scales are per row and per 32 columns: re-quantising the exact dequantised rows with the
    # search reproduces each shard's own conversion
    return L.mx_from_float(torch.cat(parts), fp4=True, search=True)


class _Nvfp4Scheme:
    """Mixed into the stock NVFP4 scheme class of one layer (see module docstring)."""

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        widths = list(getattr(layer, "logical_widths", [layer.weight_packed.shape[0]]))
        w = nvfp4_to_mx(layer.weight_packed.data, layer.weight_scale.data, layer.weight_global_scale.data, widths)
        layer.r9k_weight = w.to_tiled() if _tiled() else w
        for name in ("weight_packed", "weight_scale", "weight_global_scale", "input_global_scale"):
            if hasattr(layer, name):
                delattr(layer, name)

    def apply_weights(self, layer, x, bias=None):
        return mx_apply(layer.r9k_weight, x, bias)


class _Fp8Scheme:
    """Mixed into the stock fp8 scheme class of one layer: fp8 weights requantised to MXFP8."""

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        w8 = layer.weight.data
        s = layer.weight_scale.data.float()
        N, K = w8.shape
        wf = w8.float()
        if s.numel() == 1:
            wf = wf * s.reshape(())
        elif s.dim() == 2 and s.shape[1] == 1:  # per output channel
            wf = wf * s
        else:  # 128 x 128 blocks (ceil-divided)
            bn, bk = -(-N // s.shape[0]), -(-K // s.shape[1])
            wf = wf * s.repeat_interleave(bn, 0)[:N].repeat_interleave(bk, 1)[:, :K]
        layer.r9k_weight = L.mx_from_float(wf, fp4=False, tiled=_tiled())
        for name in ("weight", "weight_scale", "input_scale"):
            if hasattr(layer, name):
                delattr(layer, name)

    def apply_weights(self, layer, x, bias=None):
        return mx_apply(layer.r9k_weight, x, bias)


_SWAPPED: dict[type, type] = {}


def _swap(scheme, mixin: type):
    """Give this scheme instance a subclass of its own class with ``mixin`` first in the MRO."""
    base = type(scheme)
    cls = _SWAPPED.get((base, mixin))
    if cls is None:
        cls = type(f"R9k{base.__name__}", (mixin, base), {})
        _SWAPPED[(base, mixin)] = cls
    scheme.__class__ = cls
    return scheme


def served_scheme(scheme):
    """The scheme this library serves for a stock scheme instance, or the instance unchanged."""
    if scheme is None or isinstance(scheme, (_Nvfp4Scheme, _Fp8Scheme)):
        return scheme
    if isinstance(scheme, (CompressedTensorsW4A4Fp4, CompressedTensorsW4A16Fp4)) and not knobs.disabled("nvfp4"):
        return _swap(scheme, _Nvfp4Scheme)
    if (isinstance(scheme, CompressedTensorsW8A8Fp8) and not knobs.disabled("fp8")
            and not getattr(scheme, "is_static_input_scheme", False)):
        return _swap(scheme, _Fp8Scheme)
    return scheme


@register_quantization_config("compressed-tensors")
class R9kCompressedTensorsConfig(CompressedTensorsConfig):
    def get_scheme(self, layer, layer_name=None):
        return served_scheme(super().get_scheme(layer=layer, layer_name=layer_name))
