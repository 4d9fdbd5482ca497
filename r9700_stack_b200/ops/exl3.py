"""EXL3-style trellis linears on the sm_100a kernels (decode GEMV, prefill via dequantised bf16 GEMM).

``Exl3Linear`` holds one matrix (or a stack of experts of equal shape) in the trellis format of
:mod:`..quant.exl3`. Decode-width inputs (<= 16 rows per matrix) run the trellis GEMV directly
(``exl3_gemv`` partials + ``exl3_finish``); wider inputs dequantise once into a bf16 weight and use the
tcgen05 bf16 GEMM. Reference: r9700_vllm/quant/exl3_gemv.py:135-285, r9700_vllm/moe/exl3_decode.py.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native
from ..quant import exl3 as E
from . import linear as L


def _ops():
    return _native.ops()


_SCRATCH: dict[int, torch.Tensor] = {}


def scratch(device, floats: int) -> torch.Tensor:
    idx = torch.device(device).index or 0
    t = _SCRATCH.get(idx)
    if t is None or t.numel() < floats:
        t = torch.empty(max(floats, 1 << 20), dtype=torch.float32, device=device)
        _SCRATCH[idx] = t
    return t


def pick_ksplit(n_in: int, n_out: int, items: int = 1) -> int:
    """Split the input dim so that out/128 x ksplit x items CTAs fill about two waves of 148 SMs."""
    ks = 1
    while (n_out // 128) * ks * items < 296 and n_in % (128 * ks * 2) == 0 and n_in // (ks * 2) >= 256:
        ks *= 2
    return ks


@dataclass
class Exl3Linear:
    trellis: torch.Tensor  # int16 [in/16, out/16, 16K] or [E, in/16, out/16, 16K]
    suh: torch.Tensor  # f16 [in] or [E, in]
    svh: torch.Tensor  # f16 [out] or [E, out]
    K: int
    cb: int = E.MCG

    @property
    def stacked(self) -> bool:
        return self.trellis.dim() == 4

    @property
    def n_in(self) -> int:
        return self.trellis.shape[-3] * 16

    @property
    def n_out(self) -> int:
        return self.trellis.shape[-2] * 16

    @property
    def nbytes(self) -> int:
        return self.trellis.numel() * 2 + self.suh.numel() * 2 + self.svh.numel() * 2

    def dequant_bf16(self) -> L.BF16Weight:
        """The effective weight as bf16 [out, in], for wide batches (a load-time conversion). The
        tcgen05 GEMM requests its first weight tiles before waiting on the preceding kernel, so the
        stream is drained here: no GEMM may start while the dequantisation is still writing."""
        assert not self.stacked
        out = torch.empty(self.n_out, self.n_in, dtype=torch.bfloat16, device=self.trellis.device)
        _ops().exl3_dequant(self.trellis, self.suh, self.svh, self.K, self.cb, out)
        torch.cuda.current_stream(out.device).synchronize()
        return L.BF16Weight(out)

    def gemv(self, x: torch.Tensor, out: torch.Tensor, work=None, work_count=None, n_items: int = 1,
             rows: int | None = None, up: "Exl3Linear | None" = None) -> torch.Tensor:
        """out[rows] = x[rows] @ W (single matrix: rows = x.shape[0] <= 16), or per work item (expert, row0,
        rows) of a stacked matrix. With ``up``, out = silu(x W_gate) * (x W_up) (this is the gate)."""
        M = rows if rows is not None else x.shape[0]
        ks = pick_ksplit(self.n_in, self.n_out, n_items)
        MR = 8 if M <= 8 else 16
        n = ks * n_items * MR * self.n_out
        part = scratch(x.device, 2 * n if up is not None else n)
        pg = part[:n]
        o = _ops()
        o.exl3_gemv(self.trellis, self.suh, self.K, self.cb, x, M, work, work_count, n_items, ks, pg)
        pu = None
        if up is not None:
            pu = part[n:2 * n]
            o.exl3_gemv(up.trellis, up.suh, up.K, up.cb, x, M, work, work_count, n_items, ks, pu)
        o.exl3_finish(pg, pu, self.svh, up.svh if up is not None else None, ks, n_items, M, self.n_out, work,
                      work_count, out)
        return out


def random_linear(n_in: int, n_out: int, K: int, device, seed: int = 0, cb: int = E.MCG, experts: int = 0,
                  scale: float = 0.02, first: int = 0) -> Exl3Linear:
    """Random trellis weights; with ``experts`` > 0, experts first .. first + experts - 1 of a stack
    whose expert e is keyed by (seed, e), so any rank's slice of the stack is the same tensors."""
    if experts:
        parts = [E.random_pack(n_in, n_out, K, seed=seed * 1000 + e, scale=scale)
                 for e in range(first, first + experts)]
        tr = torch.stack([p[0] for p in parts]).to(device)
        suh = torch.stack([p[1] for p in parts]).to(device)
        svh = torch.stack([p[2] for p in parts]).to(device)
    else:
        tr, suh, svh = (t.to(device) for t in E.random_pack(n_in, n_out, K, seed=seed, scale=scale))
    return Exl3Linear(tr.contiguous(), suh.contiguous(), svh.contiguous(), K, cb)
