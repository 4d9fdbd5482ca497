"""Weight construction: synthetic random-init checkpoints in the named formats, and the load-time
transforms a real checkpoint goes through (NVFP4 -> MXFP4, block-fp8 -> MXFP8).

A synthetic weight is generated on the device as N(0, std) f32, quantised into the *checkpoint*
format (NVFP4 / block fp8) and then converted exactly as a loaded checkpoint tensor would be, so the
benchmark exercises the same load path a published checkpoint takes (reference: load-time
conversion in r9700_vllm/quant/nvfp4.py:78-112 and r9700_vllm/linear/fp8_block.py:23).
"""
from __future__ import annotations

import torch

from .. import knobs
from ..ops import linear as L
from ..quant import formats as F


class WeightFactory:
    def __init__(self, device, seed: int = 0, std: float = 0.02):
        self.device = torch.device(device)
        self.gen = torch.Generator(device=self.device)
        self.gen.manual_seed(seed)
        self.std = std

    def randn(self, *shape, std: float | None = None, dtype=torch.float32) -> torch.Tensor:
        t = torch.randn(*shape, generator=self.gen, device=self.device, dtype=torch.float32)
        return (t * (self.std if std is None else std)).to(dtype)

    def linear(self, N: int, K: int, fmt: str, std: float | None = None):
        """A [N, K] linear weight in device format for `fmt` (nvfp4 | mxfp4 | mxfp8 | block_fp8 | bf16)."""
        w = self.randn(N, K, std=std)
        return from_float(w, fmt)

    def norm(self, n: int, plus_one: bool) -> torch.Tensor:
        # Gemma-style norms store w with output scale (1 + w): small random offsets around zero
        if plus_one:
            return self.randn(n, std=0.1).to(torch.bfloat16)
        return (1.0 + self.randn(n, std=0.1)).to(torch.bfloat16)


def from_float(w: torch.Tensor, fmt: str, tiled: bool | None = None):
    """Quantise into `fmt`, then apply the load-time transforms (format conversion, and the
    contiguous-unit tiling of MX weights that makes every TMA box one contiguous HBM read)."""
    if tiled is None:
        tiled = knobs.get("R9K_WEIGHT_TILED") != "0"
    if fmt == "nvfp4":
        packed, s16, g = L.nvfp4_quantize(w)
        mw = L.mx_from_nvfp4(packed, s16, g, search=True)
        return mw.to_tiled() if tiled else mw
    if fmt == "mxfp4":
        return L.mx_from_float(w, fp4=True, search=True, tiled=tiled)
    if fmt == "mxfp8":
        return L.mx_from_float(w, fp4=False, tiled=tiled)
    if fmt == "block_fp8":
        # block-128 fp8 checkpoint tensor -> MXFP8 at load
        q, s = block_fp8_quantize_device(w)
        return L.mx_from_float(block_fp8_dequant_device(q, s), fp4=False, tiled=tiled)
    if fmt == "bf16":
        return L.BF16Weight(w.to(torch.bfloat16).contiguous())
    raise ValueError(f"unknown weight format {fmt}")


def block_fp8_quantize_device(w: torch.Tensor, block: int = 128):
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    pad = torch.zeros(nb * block, kb * block, device=w.device, dtype=torch.float32)
    pad[:N, :K] = w
    t = pad.view(nb, block, kb, block)
    amax = t.abs().amax(dim=(1, 3))
    s = torch.where(amax > 0, amax / F.E4M3_MAX, torch.ones_like(amax))
    q = (t / s[:, None, :, None]).clamp(-F.E4M3_MAX, F.E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(nb * block, kb * block)[:N, :K].contiguous(), s


def block_fp8_dequant_device(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    srep = s.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * srep


def weight_nbytes(w) -> int:
    if isinstance(w, L.MXWeight):
        return w.nbytes
    if isinstance(w, L.BF16Weight):
        return w.w.numel() * 2
    if isinstance(w, torch.Tensor):
        return w.numel() * w.element_size()
    return 0
