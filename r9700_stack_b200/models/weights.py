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


class TPFactory:
    """Weights of the whole (unsharded) model, each tensor drawn from its own seed and then sliced to
    this rank's tensor-parallel shard, so the model built at TP size N is exactly the TP=1 model split
    N ways (the property the multi-GPU token-equality tests check). Every rank makes the same sequence
    of calls; the call index keys the seed."""

    def __init__(self, device, seed: int, std: float):
        self.device = torch.device(device)
        self.seed = seed
        self.std = std
        self.n = 0

    def _gen(self) -> torch.Generator:
        g = torch.Generator(device=self.device)
        g.manual_seed(self.seed * 1_000_003 + 7919 * self.n)
        self.n += 1
        return g

    def full(self, *shape, std: float | None = None) -> torch.Tensor:
        """The next whole tensor, N(0, std) fp32."""
        return torch.randn(*shape, generator=self._gen(), device=self.device) * (self.std if std is None else std)

    @staticmethod
    def take_rows(full: torch.Tensor, segs) -> torch.Tensor:
        """segs = [(rows, start, count), ...]: `full` is the segments stacked along dim 0; keep rows
        [start, start + count) of each segment."""
        out, off = [], 0
        for rows, start, count in segs:
            out.append(full[off + start: off + start + count])
            off += rows
        assert off == full.shape[0], "segments must cover the whole tensor"
        return torch.cat(out) if len(out) > 1 else out[0].contiguous()

    @staticmethod
    def _checkpoint(full: torch.Tensor, fmt: str):
        """Block-fp8 checkpoints are quantised in 128x128 blocks of the whole tensor, whose borders
        need not fall on shard borders: quantise the whole tensor, then cut the shard from its exact
        dequantisation (what a loader of such a checkpoint does before requantising to MXFP8)."""
        if fmt == "block_fp8":
            q, s = block_fp8_quantize_device(full)
            return block_fp8_dequant_device(q, s), "mxfp8"
        return full, fmt

    def rows(self, segs, K: int, fmt: str, std: float | None = None):
        """A row-parallel shard (column-parallel linear: output features split) in format `fmt`."""
        full, f2 = self._checkpoint(self.full(sum(s[0] for s in segs), K, std=std), fmt)
        return from_float(self.take_rows(full, segs), f2, global_from=full)

    def cols(self, N: int, K: int, start: int, count: int, fmt: str, std: float | None = None):
        """A column shard (row-parallel linear: input features split) in format `fmt`."""
        full, f2 = self._checkpoint(self.full(N, K, std=std), fmt)
        return from_float(full[:, start:start + count].contiguous(), f2, global_from=full)

    def raw_rows(self, segs, *rest, std: float | None = None, dtype=torch.float32) -> torch.Tensor:
        full = self.full(sum(s[0] for s in segs), *rest, std=std)
        return self.take_rows(full, segs).to(dtype)


def from_float(w: torch.Tensor, fmt: str, tiled: bool | None = None, global_from: torch.Tensor | None = None):
    """Quantise into `fmt`, then apply the load-time transforms (format conversion, and the
    contiguous-unit tiling of MX weights that makes every TMA box one contiguous HBM read).
    ``global_from``: the whole tensor a shard was cut from; NVFP4's per-tensor global scale is taken
    from it, as a checkpoint stores one global scale per (unsharded) tensor."""
    tiled_forced = tiled is True  # grouped expert stacks need the MX tiled layout
    if tiled is None:
        tiled = knobs.get("R9K_WEIGHT_TILED") != "0"
    if fmt == "nvfp4":
        gs = F.nvfp4_global_scale(global_from.float()) if global_from is not None else None
        packed, s16, g = L.nvfp4_quantize(w, global_scale=gs)
        if knobs.get("R9K_NVFP4") == "native" and w.shape[1] % 64 == 0 and not tiled_forced:
            return L.NVF4Weight.from_checkpoint(packed, s16, g)
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
    if isinstance(w, (L.MXWeight, L.NVF4Weight)):
        return w.nbytes
    if isinstance(w, L.BF16Weight):
        return w.w.numel() * 2
    if isinstance(w, torch.Tensor):
        return w.numel() * w.element_size()
    return 0
