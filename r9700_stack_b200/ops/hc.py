"""Hyper-connections (Flash-Next / Qwen4Exp class): HC residual streams around every block.

The residual X [T, HC * H] holds HC copies of the hidden state. At every norm point (before each
mixer, each FFN and the LM head):

1. the previous block's output y [T, H] is injected into every stream with a per-token weight
   ``2 sigmoid(l_s / HC)``, ``l = y W_l^T`` ([T, HC], one small GEMM), and every stream is
   RMS-normalised with its own weight (``hc_combine_norm``);
2. the next block's input is the sigmoid-gated mean of the normalised streams (``hc_gate_mix``)
   with a learned gate vector per norm point.

``combine_norm_ref`` / ``gate_mix_ref`` restate both kernels in torch with the same rounding
points. Reference: kernels/r9k_hc.hip:4-14 (formulas), r9700_vllm/models/qwen4_exp.py (model glue).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native
from . import linear as L


@dataclass
class HCPoint:
    """Parameters of one norm point: per-stream norm weight [HC * H], gate vector [1, HC * H] and
    the injection-logit projection [HC, H]."""

    w: torch.Tensor
    g: torch.Tensor
    wl: L.BF16Weight


def random_point(wf, HC: int, H: int) -> HCPoint:
    return HCPoint(
        w=wf.randn(HC * H, std=0.1, dtype=torch.bfloat16),
        g=wf.randn(1, HC * H, std=1.0, dtype=torch.bfloat16),
        wl=L.BF16Weight(wf.randn(HC, H, std=0.05, dtype=torch.bfloat16)),
    )


def combine_norm(res, block, l, w, HC: int, eps: float, out) -> None:
    _native.ops().hc_combine_norm(res, block, l, w, HC, float(eps), out)


def gate_mix(x, g, HC: int, out) -> None:
    _native.ops().hc_gate_mix(x, g, HC, out)


def point(res, y, p: HCPoint, HC: int, eps: float, out) -> None:
    """Fused norm point (injection logits, residual update, per-stream norm, gated mix) in one launch."""
    _native.ops().hc_point(res, y, p.wl.w, p.w, p.g, HC, float(eps), out)


def point_ref(res, y, p: HCPoint, HC: int, eps: float):
    """(new residual, next block input) of a norm point, in torch."""
    l = y.float() @ p.wl.w.float().T if y is not None else None
    r, n = combine_norm_ref(res, y, l, p.w, HC, eps)
    return r, gate_mix_ref(n, p.g, HC)


def combine_norm_ref(res, block, l, w, HC: int, eps: float):
    """(new residual, normalised streams), both bf16, as the kernel computes them."""
    T, D = res.shape
    H = D // HC
    r = res.float().view(T, HC, H)
    if block is not None:
        inj = 2 * torch.sigmoid(l.float() / HC)  # [T, HC]
        r = (r + block.float()[:, None, :] * inj[:, :, None]).bfloat16().float()
    rr = torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps)
    wv = w.float().view(HC, H) if w.numel() == D else w.float().view(1, H)
    y = r * rr
    y = (y + y * wv[None]).bfloat16()
    return r.bfloat16().view(T, D), y.view(T, D)


def gate_mix_ref(x, g, HC: int):
    T, D = x.shape
    H = D // HC
    gg = g.float().expand(T, D).view(T, HC, H)
    return ((torch.sigmoid(gg) * x.float().view(T, HC, H)).sum(1) / HC).bfloat16()
