"""Embedding tables resident in pinned host memory, gathered by the GPU through their UVA mapping.

``HostTable`` holds a [rows, row_bytes] uint8 table in page-locked host memory in one of two row
formats (``int6`` fused rows with fp16 scales per 32, or ``fp8`` e4m3 with ue8m0 scales per 32) and
gathers rows into a device bf16 buffer with one kernel (``host_gather``), so it runs inside CUDA
graphs. Used for the Flash-Next per-layer embeddings and the DeepSeek Engram n-gram tables, which do
not fit in HBM at their published sizes. Reference: r9700_vllm/utils/hostmem.py:18-61,
r9700_vllm/ple/int6.py:35-171, kernels/r9k_ple.hip.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _native

FMT = {"int6": 0, "fp8": 1}


def int6_row_bytes(dim: int) -> int:
    return dim * 6 // 8 + dim // 32 * 2


def fp8_row_bytes(dim: int) -> int:
    return dim + dim // 32


def quantize_int6(x: torch.Tensor) -> torch.Tensor:
    """[rows, dim] float -> uint8 [rows, int6_row_bytes(dim)] (codes + fp16 scales), CPU."""
    rows, dim = x.shape
    g = x.float().view(rows, dim // 32, 32)
    s = (g.abs().amax(-1) / 31.0).clamp(min=1e-8).to(torch.float16)
    q = torch.round(g / s.float()[..., None]).clamp(-31, 31).to(torch.int64).view(rows, dim) + 32
    q4 = q.view(rows, dim // 4, 4)
    word = q4[..., 0] | (q4[..., 1] << 6) | (q4[..., 2] << 12) | (q4[..., 3] << 18)
    b = torch.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], -1).to(torch.uint8).view(rows, -1)
    sb = s.view(torch.uint8).view(rows, -1)
    return torch.cat([b, sb], 1).contiguous()


def dequant_int6(rows_u8: torch.Tensor, dim: int) -> torch.Tensor:
    n = rows_u8.shape[0]
    b = rows_u8[:, : dim * 6 // 8].to(torch.int64).view(n, dim // 4, 3)
    word = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    codes = torch.stack([(word >> (6 * k)) & 63 for k in range(4)], -1).view(n, dim) - 32
    s = rows_u8[:, dim * 6 // 8:].contiguous().view(torch.float16).float()
    return codes.float() * s.repeat_interleave(32, 1)


def quantize_fp8(x: torch.Tensor) -> torch.Tensor:
    rows, dim = x.shape
    g = x.float().view(rows, dim // 32, 32)
    amax = g.abs().amax(-1).clamp(min=2.0 ** -120)
    e = torch.ceil(torch.log2(amax / 448.0)).clamp(-127, 127)
    q = (g / torch.exp2(e)[..., None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8).view(rows, dim)
    return torch.cat([q, (e + 127).to(torch.uint8)], 1).contiguous()


def dequant_fp8(rows_u8: torch.Tensor, dim: int) -> torch.Tensor:
    q = rows_u8[:, :dim].contiguous().view(torch.float8_e4m3fn).float()
    e = rows_u8[:, dim:].float() - 127
    return q * torch.exp2(e).repeat_interleave(32, 1)


class HostTable:
    def __init__(self, rows: int, dim: int, fmt: str = "int6"):
        assert fmt in FMT and dim % 32 == 0
        self.rows, self.dim, self.fmt = rows, dim, fmt
        rb = int6_row_bytes(dim) if fmt == "int6" else fp8_row_bytes(dim)
        self.table = torch.empty(rows, rb, dtype=torch.uint8, pin_memory=True)

    @classmethod
    def random(cls, rows: int, dim: int, fmt: str = "int6", seed: int = 0, std: float = 0.02, chunk: int = 1 << 20):
        """Synthetic table: N(0, std) rows quantised into the format, written in chunks."""
        t = cls(rows, dim, fmt)
        g = torch.Generator().manual_seed(seed)
        for r0 in range(0, rows, chunk):
            n = min(chunk, rows - r0)
            x = torch.randn(n, dim, generator=g) * std
            t.table[r0:r0 + n] = quantize_int6(x) if fmt == "int6" else quantize_fp8(x)
        return t

    @property
    def nbytes(self) -> int:
        return self.table.numel()

    def gather(self, ids: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """ids: device int64 [n]; out: device bf16 [n, dim]."""
        _native.ops().host_gather(self.table, ids, FMT[self.fmt], self.dim, out)
        return out

    def gather_ref(self, ids: torch.Tensor) -> torch.Tensor:
        idx = ids.cpu().long()
        ok = (idx >= 0) & (idx < self.rows)
        rows = self.table[idx.clamp(0, self.rows - 1)]
        v = dequant_int6(rows, self.dim) if self.fmt == "int6" else dequant_fp8(rows, self.dim)
        return v * ok[:, None].float()


def ngram_ids(tokens: torch.Tensor, order: int, rows: int, salt: int = 0) -> torch.Tensor:
    """Hash of each position's last ``order`` tokens into [0, rows) (multiplicative, order-sensitive);
    tokens [T] int64 of one sequence. Positions with fewer predecessors hash the available ones."""
    h = torch.zeros_like(tokens) + (salt * 0x9E3779B1 + order)
    for j in range(order):
        prev = torch.roll(tokens, j)
        if j:
            prev[:j] = 0
        h = (h * 1000003 + prev + 1) & 0x7FFFFFFFFFFF
    return h % rows
