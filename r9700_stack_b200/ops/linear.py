"""Linear layers on the tcgen05 GEMM core.

Weights are held in one of three device formats:

* ``MXWeight(fp4=True)``  - MXFP4: packed e2m1 [N, K/2] + ue8m0 scales per 32 (chunk layout).
  NVFP4 checkpoints convert to this at load (MSE-searched exponents), as the reference does
  (r9700_vllm/quant/nvfp4.py:78-112).
* ``MXWeight(fp4=False)`` - MXFP8: e4m3 [N, K] + ue8m0 scales per 32. Block-128 fp8 and per-row fp8
  checkpoints (lm heads, drafters) convert to this at load.
* ``BF16Weight``           - unquantised weights.

Activations feeding MX weights are MXFP8 (``MXAct``), produced directly by the fused
RMSNorm/SwiGLU epilogues, or by :func:`quant_act` for other producers.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native
from ..quant import formats as F
from ..utils import status as _status


def _ops():
    return _native.ops()


_WS: dict[int, torch.Tensor] = {}
SK_WORKSPACE_FLOATS = 65536 + 4 * 148 * 2 * 2 * 64 * 128 + 4096


def gemm_workspace(device) -> torch.Tensor | None:
    """Per-device fp32 scratch of the split-K / stream-K decode GEMMs: 65536 per-tile arrival counters
    (kept at zero between calls by the kernels themselves) followed by partial-tile slots. GEMMs that
    share it must run in stream order (one stream per device)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _WS.get(idx)
    if t is None:
        t = torch.zeros(SK_WORKSPACE_FLOATS, dtype=torch.float32, device=f"cuda:{idx}")
        _WS[idx] = t
    return t


def sf_bytes(rows: int, K: int) -> int:
    return F.sf_num_bytes(rows, K // 32)


@dataclass
class MXWeight:
    """MX weight. ``q`` is row-major [N, K/2 | K], or pre-tiled [units, 128, 64 | 128] where unit
    (t, kc) = rows 128t..128t+127 x K elements 128kc..128kc+127 is contiguous (rows padded to 128):
    one TMA box is then one contiguous HBM read. The scale chunks use the same unit order."""

    q: torch.Tensor
    sf: torch.Tensor  # uint8 chunk layout
    fp4: bool
    N: int
    K: int

    @property
    def tiled(self) -> bool:
        return self.q.dim() == 3

    @property
    def nbytes(self) -> int:
        return self.q.numel() + self.sf.numel()

    def rowmajor_q(self) -> torch.Tensor:
        if not self.tiled:
            return self.q
        cb = self.q.shape[-1]
        kch = self.K // 128
        rt = self.q.shape[0] // kch
        return self.q.view(rt, kch, 128, cb).permute(0, 2, 1, 3).reshape(rt * 128, kch * cb)[: self.N].contiguous()

    def to_tiled(self) -> "MXWeight":
        if self.tiled:
            return self
        cb = 64 if self.fp4 else 128
        kch = self.K // 128
        rt = (self.N + 127) // 128
        q = self.q
        if rt * 128 != self.N:
            q = torch.cat([q, torch.zeros(rt * 128 - self.N, q.shape[1], dtype=q.dtype, device=q.device)], 0)
        t = q.view(rt, 128, kch, cb).permute(0, 2, 1, 3).contiguous().view(rt * kch, 128, cb)
        return MXWeight(t, self.sf, self.fp4, self.N, self.K)

    def dequant(self) -> torch.Tensor:
        out = torch.empty(self.N, self.K, dtype=torch.float32, device=self.q.device)
        _ops().dequant_mx(self.rowmajor_q(), self.sf, self.fp4, out)
        return out

    def narrow_rows(self, start: int, length: int) -> "MXWeight":
        """Row slice (start and length multiples of 128 so that scale chunks stay whole)."""
        assert start % 128 == 0 and (length % 128 == 0 or start + length == self.N)
        kchunks = (self.K // 32 + 3) // 4
        c0 = (start // 128) * kchunks * 512
        c1 = ((start + length + 127) // 128) * kchunks * 512
        if self.tiled:
            kch = self.K // 128
            q = self.q[(start // 128) * kch : ((start + length + 127) // 128) * kch]
        else:
            q = self.q[start : start + length]
        return MXWeight(q, self.sf[c0:c1], self.fp4, length, self.K)


@dataclass
class BF16Weight:
    w: torch.Tensor  # bf16 [N, K]

    @property
    def N(self) -> int:
        return self.w.shape[0]

    @property
    def K(self) -> int:
        return self.w.shape[1]


@dataclass
class NVF4Weight:
    """NVFP4 weight served without conversion (``R9K_NVFP4=native``): the checkpoint's e2m1 codes and
    e4m3 block-16 scales, re-laid out into [N/128][K/64] units of 128 rows x 64 elements (4 KiB of
    codes ``q``, 512 B of scales ``s``), and alpha = 1 / global scale. ``gemm_nvf4`` expands units to
    bf16 on chip (exact) and multiplies bf16 activations."""

    q: torch.Tensor  # uint8 [N/128 * K/64, 128, 32]
    s: torch.Tensor  # uint8 [N/128 * K/64, 128, 4]
    alpha: float
    N: int
    K: int

    @property
    def nbytes(self) -> int:
        return self.q.numel() + self.s.numel()

    @staticmethod
    def from_checkpoint(packed: torch.Tensor, s16: torch.Tensor, g: float) -> "NVF4Weight":
        """packed [N, K/2] (low nibble = even element), s16 [N, K/16] e4m3 bytes, global scale g.
        Rows are padded to a multiple of 128 with zero codes and scales (the kernel masks them)."""
        N, K = packed.shape[0], packed.shape[1] * 2
        assert K % 64 == 0, "native NVFP4 needs K % 64 == 0"
        Np = -(-N // 128) * 128
        packed, s16 = packed.contiguous(), s16.contiguous().view(torch.uint8)
        if Np != N:
            packed = torch.cat([packed, packed.new_zeros(Np - N, packed.shape[1])])
            s16 = torch.cat([s16, s16.new_zeros(Np - N, s16.shape[1])])
        q = packed.view(Np // 128, 128, K // 64, 32).permute(0, 2, 1, 3).reshape(-1, 128, 32).contiguous()
        s = s16.view(Np // 128, 128, K // 64, 4).permute(0, 2, 1, 3)
        return NVF4Weight(q, s.reshape(-1, 128, 4).contiguous(), 1.0 / float(g), N, K)

    def dequant(self) -> torch.Tensor:
        """fp32 [N, K] (the exact checkpoint values)."""
        from ..quant import formats as F

        N, K = self.N, self.K
        Np = -(-N // 128) * 128
        packed = self.q.view(Np // 128, K // 64, 128, 32).permute(0, 2, 1, 3).reshape(Np, K // 2)[:N]
        s16 = self.s.view(Np // 128, K // 64, 128, 4).permute(0, 2, 1, 3).reshape(Np, K // 16)[:N]
        return F.dequant_nvfp4(packed.cpu(), s16.cpu(), 1.0 / self.alpha).to(self.q.device)


@dataclass
class MXAct:
    q: torch.Tensor  # uint8 [M, K] e4m3
    sf: torch.Tensor  # uint8 chunk layout (rows padded to 128)

    @property
    def M(self) -> int:
        return self.q.shape[0]

    def narrow(self, m: int) -> "MXAct":
        return MXAct(self.q[:m], self.sf)


def act_sf_bytes(M: int, K: int) -> int:
    """Activation scale buffers cover the token count rounded up to 256 (the widest GEMM tile)."""
    return sf_bytes(max(256, (M + 255) // 256 * 256), K)


def alloc_act(M: int, K: int, device) -> MXAct:
    return MXAct(
        torch.empty(M, K, dtype=torch.uint8, device=device),
        torch.zeros(act_sf_bytes(M, K), dtype=torch.uint8, device=device),
    )


# ------------------------------------------------------------------------------------------------
# weight construction
# ------------------------------------------------------------------------------------------------
def mx_from_float(w: torch.Tensor, fp4: bool = True, search: bool = True, tiled: bool = False) -> MXWeight:
    """Quantise a float weight [N, K] on the device (f32 staging, one matrix at a time)."""
    N, K = w.shape
    dev = w.device
    wf = w.float().contiguous()
    sf = torch.zeros(sf_bytes(N, K), dtype=torch.uint8, device=dev)
    if fp4:
        q = torch.empty(N, K // 2, dtype=torch.uint8, device=dev)
        _ops().quant_weight_mxfp4(wf, q, sf, search)
    else:
        q = torch.empty(N, K, dtype=torch.uint8, device=dev)
        _ops().quant_weight_mxfp8(wf, q, sf)
    mw = MXWeight(q, sf, fp4, N, K)
    return mw.to_tiled() if tiled else mw


def nvfp4_quantize(w: torch.Tensor, global_scale: float | None = None):
    """float [N, K] -> NVFP4 (packed, s16 e4m3 bytes, g) on the device."""
    N, K = w.shape
    wf = w.float().contiguous()
    g = F.nvfp4_global_scale(wf) if global_scale is None else global_scale
    packed = torch.empty(N, K // 2, dtype=torch.uint8, device=w.device)
    s16 = torch.empty(N, K // 16, dtype=torch.uint8, device=w.device)
    _ops().quant_weight_nvfp4(wf, float(g), packed, s16)
    return packed, s16, float(g)


def mx_from_nvfp4(packed: torch.Tensor, s16: torch.Tensor, g: float, search: bool = True) -> MXWeight:
    N, K2 = packed.shape
    K = K2 * 2
    sf = torch.zeros(sf_bytes(N, K), dtype=torch.uint8, device=packed.device)
    out = torch.empty(N, K2, dtype=torch.uint8, device=packed.device)
    _ops().nvfp4_to_mxfp4(packed.contiguous(), s16.contiguous(), float(g), out, sf, search)
    return MXWeight(out, sf, True, N, K)


# ------------------------------------------------------------------------------------------------
# activations and GEMMs
# ------------------------------------------------------------------------------------------------
def quant_act(x: torch.Tensor, out: MXAct | None = None) -> MXAct:
    M, K = x.shape
    if out is None:
        out = alloc_act(M, K, x.device)
    _ops().quant_act_mxfp8(x, out.q, out.sf)
    return out


def rmsnorm(
    x: torch.Tensor,
    w: torch.Tensor,
    eps: float,
    *,
    plus_one: bool = False,
    residual: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    quant_out: MXAct | None = None,
) -> None:
    """Fused (residual add) + RMSNorm (+ MXFP8 quant). Writes into the given outputs."""
    _ops().rmsnorm_quant(
        x,
        residual,
        residual_out,
        w,
        float(eps),
        bool(plus_one),
        out,
        quant_out.q if quant_out is not None else None,
        quant_out.sf if quant_out is not None else None,
    )


def mx_linear(
    x: MXAct,
    w: MXWeight,
    out: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    alpha: float = 1.0,
    out_dtype=torch.bfloat16,
) -> torch.Tensor:
    M = x.M
    if out is None:
        out = torch.empty(M, w.N, dtype=out_dtype, device=x.q.device)
    _ops().gemm_mx(w.q, w.sf, w.fp4, x.q, x.sf, out, residual, float(alpha), _status.status(x.q.device),
                   gemm_workspace(x.q.device))
    return out


SWIGLU_SPLIT_M = 256  # from this many tokens on, gate / up run as two GEMMs + one SwiGLU-quant pass


def mx_swiglu(x: MXAct, w_gate: MXWeight, w_up: MXWeight, out: MXAct | None = None) -> MXAct:
    """silu(x W_gate^T) * (x W_up^T) as MXFP8. Decode-sized M: one dual-accumulator kernel with the
    SwiGLU and the quantisation in its epilogue. Prefill-sized M: the gate and up GEMMs at full tile
    width into one bf16 buffer, then swiglu_quant_mxfp8 (measured at 17408 x 5120, M = 8192: the dual
    kernel 3.87 ms, 0.76 PFLOP/s; one wide GEMM 1.06 ms)."""
    M = x.M
    if out is None:
        out = alloc_act(M, w_gate.N, x.q.device)
    if M >= SWIGLU_SPLIT_M and w_gate.N % 32 == 0 and not torch.cuda.is_current_stream_capturing():
        N = w_gate.N
        gu = _swiglu_scratch(M, N, x.q.device)
        mx_linear(x, w_gate, out=gu[0])
        mx_linear(x, w_up, out=gu[1])
        _ops().swiglu_quant_mxfp8(gu[0], gu[1], out.q, out.sf)
        return out
    _ops().gemm_mx_swiglu(
        w_gate.q, w_gate.sf, w_up.q, w_up.sf, w_gate.fp4, x.q, x.sf, out.q, out.sf, _status.status(x.q.device),
        gemm_workspace(x.q.device),
    )
    return out


_SWIGLU_BUF: dict = {}


def _swiglu_scratch(M: int, N: int, device) -> torch.Tensor:
    """[2, M, N] bf16 gate / up outputs of the split SwiGLU path, reused across calls (eager prefill)."""
    key = torch.device(device)
    buf = _SWIGLU_BUF.get(key)
    if buf is None or buf.numel() < 2 * M * N:
        buf = torch.empty(2 * M * N, dtype=torch.bfloat16, device=key)
        _SWIGLU_BUF[key] = buf
    return buf[: 2 * M * N].view(2, M, N)


def bf16_linear(
    x: torch.Tensor, w: BF16Weight, out: torch.Tensor | None = None, residual: torch.Tensor | None = None,
    alpha: float = 1.0, out_dtype=torch.bfloat16,
) -> torch.Tensor:
    M = x.shape[0]
    if out is None:
        out = torch.empty(M, w.N, dtype=out_dtype, device=x.device)
    _ops().gemm_bf16(w.w, x, out, residual, float(alpha), _status.status(x.device), gemm_workspace(x.device))
    return out


def bf16_swiglu(x: torch.Tensor, w_gate: BF16Weight, w_up: BF16Weight, out: torch.Tensor | None = None):
    """silu(x W_gate^T) * (x W_up^T) in one tcgen05 kernel (bf16 weights, bf16 result)."""
    if out is None:
        out = torch.empty(x.shape[0], w_gate.N, dtype=torch.bfloat16, device=x.device)
    _ops().gemm_bf16_swiglu(w_gate.w, w_up.w, x, out, _status.status(x.device), gemm_workspace(x.device))
    return out


def nvf4_linear(x: torch.Tensor, w: NVF4Weight, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = x @ W^T for bf16 x and a native NVFP4 weight."""
    if out is None:
        out = torch.empty(x.shape[0], w.N, dtype=torch.bfloat16, device=x.device)
    _ops().gemm_nvf4(w.q, w.s, w.alpha, None, None, 1.0, x, out, _status.status(x.device))
    return out


def nvf4_swiglu(x: torch.Tensor, w_gate: NVF4Weight, w_up: NVF4Weight, out: torch.Tensor | None = None):
    """silu(x W_gate^T) * (x W_up^T) in one kernel (native NVFP4 weights, bf16 in and out)."""
    if out is None:
        out = torch.empty(x.shape[0], w_gate.N, dtype=torch.bfloat16, device=x.device)
    _ops().gemm_nvf4(w_gate.q, w_gate.s, w_gate.alpha, w_up.q, w_up.s, w_up.alpha, x, out, _status.status(x.device))
    return out


def stack_experts(ws: list[MXWeight]) -> MXWeight:
    """Stack per-expert MX weights [N, K] into one [E * N, K] matrix (pre-tiled units, scale chunks
    concatenated in the same order) for the grouped GEMM."""
    assert all(w.N == ws[0].N and w.K == ws[0].K and w.fp4 == ws[0].fp4 for w in ws) and ws[0].N % 128 == 0
    tiled = [w.to_tiled() for w in ws]
    q = torch.cat([w.q for w in tiled], 0)
    sf = torch.cat([w.sf for w in tiled], 0)
    return MXWeight(q, sf, ws[0].fp4, ws[0].N * len(ws), ws[0].K)
