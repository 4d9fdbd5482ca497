"""Manifold hyper-connections (DeepSeek-V4 class): the seam op and a PyTorch restatement.

``MHC`` holds one sublayer's parameters (fn [24, 4H] fp32, scale [3], base [24]) and runs the two-launch
seam kernel of ``csrc/mhc.cu``: fold the previous sublayer's output into the 4 residual streams with
its post/comb mixes, then compute this sublayer's mixes and its input. ``mhc_seam_ref`` states the
same computation in PyTorch (the semantics of vLLM's ``mhc_post_torch`` + ``mhc_pre_torch``).
Reference: r9700_vllm/hc_dsv4.py:169-265, kernels/r9k_mhc.hip:144-303.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native

HC, NMIX = 4, 24


@dataclass
class MHCParams:
    fn: torch.Tensor  # [24, 4H] fp32
    scale: torch.Tensor  # [3] fp32
    base: torch.Tensor  # [24] fp32
    rms_eps: float = 1e-6
    pre_eps: float = 1e-2
    sk_eps: float = 1e-6
    post_mult: float = 2.0
    sk_repeat: int = 20


def seam(R: torch.Tensor, p: MHCParams, so=None, post_in=None, comb_in=None, R_out=None, post_out=None,
         comb_out=None, li=None, part=None):
    """R [T, 4, H] bf16 -> (R_out, post [T, 4], comb [T, 4, 4], li [T, H]); so/post_in/comb_in fold the
    previous sublayer in (None: R_out = R)."""
    T, _, H = R.shape
    dev = R.device
    R_out = R if R_out is None else R_out
    post_out = torch.empty(T, HC, device=dev) if post_out is None else post_out
    comb_out = torch.empty(T, HC, HC, device=dev) if comb_out is None else comb_out
    li = torch.empty(T, H, dtype=torch.bfloat16, device=dev) if li is None else li
    part = torch.empty(T * (H // 64) * (NMIX + 1), device=dev) if part is None else part
    _native.ops().mhc_seam(R, so, post_in, comb_in, p.fn, p.scale, p.base, p.rms_eps, p.pre_eps, p.sk_eps,
                           p.post_mult, p.sk_repeat, R_out, post_out, comb_out, li, part)
    return R_out, post_out, comb_out, li


def seam_ref(R: torch.Tensor, p: MHCParams, so=None, post_in=None, comb_in=None):
    """PyTorch restatement (fp32 math, bf16 storage of R' and li)."""
    Rf = R.float()
    if so is not None:
        Rf = (torch.einsum("tij,tih->tjh", comb_in.float(), Rf) + post_in.float()[..., None] * so.float()[:, None, :])
        Rf = Rf.to(torch.bfloat16).float()
    T, _, H = Rf.shape
    x = Rf.reshape(T, HC * H)
    mixes = x @ p.fn.t()
    mixes = mixes * torch.rsqrt(x.square().sum(-1, keepdim=True) / (HC * H) + p.rms_eps)
    pre = torch.sigmoid(mixes[:, :HC] * p.scale[0] + p.base[:HC]) + p.pre_eps
    post = torch.sigmoid(mixes[:, HC:2 * HC] * p.scale[1] + p.base[HC:2 * HC]) * p.post_mult
    c = mixes[:, 2 * HC:].view(T, HC, HC) * p.scale[2] + p.base[2 * HC:].view(1, HC, HC)
    c = torch.softmax(c, -1) + p.sk_eps
    c = c / (c.sum(-2, keepdim=True) + p.sk_eps)
    for _ in range(p.sk_repeat - 1):
        c = c / (c.sum(-1, keepdim=True) + p.sk_eps)
        c = c / (c.sum(-2, keepdim=True) + p.sk_eps)
    li = (pre[..., None] * Rf).sum(1).to(torch.bfloat16)
    return Rf.to(torch.bfloat16), post, c, li
