"""Plain-PyTorch oracle of the lossy compressed all-reduce (WHT-64 rotation, 4/6-bit codes).

The kernel (``symm_ar_wht`` in ``csrc/collectives.cu``) rotates every 64-element block by an
orthonormal 64-point Walsh-Hadamard transform, stores a bf16 scale ``amax / qmax`` and
round-to-nearest-even integer codes in [-qmax, qmax] (qmax = 7 for 4 bits, 31 for 6 bits), sums the
ranks' dequantised codes in rank order in fp32 in the rotated domain and rotates back. This module
restates those steps with the same butterfly order, so on the same inputs it reproduces the
kernel's output bit for bit. Reference: kernels/r9k_ar_wht.hip:4-27 (two-rank WHT wire),
kernels/r9k_ar4.hip:1-42 (reduction in the rotated domain, bit-identical ranks).
"""
from __future__ import annotations

import torch

BLOCK = 64


def wht64(y: torch.Tensor) -> torch.Tensor:
    """Orthonormal WHT over the last dim (64), butterflies at strides 1, 2, ..., 32 in that order."""
    y = y.float().clone()
    lead = y.shape[:-1]
    s = 1
    while s < BLOCK:
        v = y.reshape(*lead, BLOCK // (2 * s), 2, s)
        lo, hi = v[..., 0, :], v[..., 1, :]
        y = torch.stack([lo + hi, lo - hi], dim=-2).reshape(*lead, BLOCK)
        s *= 2
    return y * 0.125


def quantize(x: torch.Tensor, bits: int) -> tuple[torch.Tensor, torch.Tensor]:
    """x [n] (n % 64 == 0) -> (codes int8 [n/64, 64], scales fp32 [n/64] holding bf16 values)."""
    qmax = (1 << (bits - 1)) - 1
    y = wht64(x.float().reshape(-1, BLOCK))
    amax = y.abs().amax(-1)
    s = (amax / qmax).to(torch.bfloat16).float()
    inv = torch.where(s > 0, 1.0 / s, torch.zeros_like(s))
    q = torch.round(y * inv[:, None]).clamp(-qmax, qmax).to(torch.int8)
    return q, s


def all_reduce_ref(xs: list[torch.Tensor], bits: int) -> torch.Tensor:
    """The compressed all-reduce of the ranks' inputs xs (rank order), as the kernel computes it."""
    acc = None
    for x in xs:
        q, s = quantize(x, bits)
        t = q.float() * s[:, None]
        acc = t if acc is None else acc + t
    return wht64(acc).to(torch.bfloat16).reshape(xs[0].shape)


def wire_bytes(n: int, bits: int) -> int:
    """Bytes one rank publishes for n elements (codes + one bf16 scale per 64)."""
    return n // BLOCK * (8 * bits + 2)
