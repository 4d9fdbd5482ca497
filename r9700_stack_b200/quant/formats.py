"""Pure-torch CPU oracle for every weight / activation format the framework handles.

These functions define the numerics; the CUDA kernels are tested against them bit for bit where the
math is exact (packing, scale choice, dequantisation) and within fp32 accumulation tolerance for
GEMMs.

Formats
-------
* **e2m1 (fp4)**: sign + 2-bit exponent + 1-bit mantissa; magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}. Two
  codes per byte, element ``2i`` in the low nibble.
* **MXFP4 / MXFP8**: e2m1 / e4m3 values with one ue8m0 (power-of-two, bias 127) scale per 32 elements
  along K. The scale exponent is ``ceil(log2(amax / qmax))`` (no clipping); MXFP4 weights can search
  exponent shifts -2..+2 for the lowest squared error.
* **NVFP4**: e2m1 values, one e4m3 scale per 16 elements, one fp32 global scale ``g``:
  ``w = v * s / g`` (reference: r9700_vllm/quant/nvfp4.py:39).
* **Block-128 fp8**: e4m3 weights with an fp32 scale per 128x128 block (reference:
  r9700_vllm/linear/fp8_block.py:23).
* **Per-token fp8**: e4m3 rows with scale ``amax / 448`` (reference: kernels/r9k_moe_mxfp4a8.hip:1745).

Scale-factor layout (``sf_offsets``)
------------------------------------
MX scales are stored in 512-byte chunks, one chunk per (128 rows) x (4 scale blocks = 128 K
elements), chunks ordered ``[row // 128][kblock // 4]``. Inside a chunk the byte for row ``r`` and
k-block ``j`` sits at ``(r % 32) * 16 + ((r % 128) // 32) * 4 + j % 4``. This is the layout the
tensor core's block-scaled MMA reads from TMEM after a ``tcgen05.cp 32x128b.warpx4``, so kernels
copy chunks without rearranging them.
"""
from __future__ import annotations

import math

import torch

E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)
FP4_MAX = 6.0
E4M3_MAX = 448.0


# ------------------------------------------------------------------------------------------------
# scale-factor layout
# ------------------------------------------------------------------------------------------------
def sf_num_bytes(rows: int, kblocks: int) -> int:
    return ((rows + 127) // 128) * ((kblocks + 3) // 4) * 512


def sf_offsets(rows: int, kblocks: int) -> torch.Tensor:
    r = torch.arange(rows, dtype=torch.int64)[:, None]
    j = torch.arange(kblocks, dtype=torch.int64)[None, :]
    kchunks = (kblocks + 3) // 4
    chunk = (r >> 7) * kchunks + (j >> 2)
    return chunk * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (j & 3)


def pack_sf(e_biased: torch.Tensor) -> torch.Tensor:
    """[rows, kblocks] uint8 biased exponents -> flat chunk-layout uint8 buffer (padding zero)."""
    rows, kb = e_biased.shape
    out = torch.zeros(sf_num_bytes(rows, kb), dtype=torch.uint8)
    out[sf_offsets(rows, kb).reshape(-1)] = e_biased.reshape(-1).to(torch.uint8).cpu()
    return out


def unpack_sf(flat: torch.Tensor, rows: int, kblocks: int) -> torch.Tensor:
    return flat.cpu()[sf_offsets(rows, kblocks).reshape(-1)].reshape(rows, kblocks)


# ------------------------------------------------------------------------------------------------
# scalar formats
# ------------------------------------------------------------------------------------------------
def e2m1_encode(v: torch.Tensor) -> torch.Tensor:
    """Round to nearest e2m1 (ties to even code), saturating at 6. Returns uint8 codes 0..15."""
    a = v.abs().float()
    code = (
        (a > 0.25).to(torch.uint8)
        + (a >= 0.75).to(torch.uint8)
        + (a > 1.25).to(torch.uint8)
        + (a >= 1.75).to(torch.uint8)
        + (a > 2.5).to(torch.uint8)
        + (a >= 3.5).to(torch.uint8)
        + (a > 5.0).to(torch.uint8)
    )
    neg = (v < 0) & (code != 0)
    return code | (neg.to(torch.uint8) << 3)


def e2m1_decode(code: torch.Tensor) -> torch.Tensor:
    c = code.to(torch.int64)
    mag = E2M1_VALUES.to(code.device)[c & 7]
    return torch.where((c & 8) != 0, -mag, mag)


def pack_fp4(codes: torch.Tensor) -> torch.Tensor:
    """[..., K] codes -> [..., K/2] bytes, element 2i in the low nibble."""
    c = codes.to(torch.uint8)
    return c[..., 0::2] | (c[..., 1::2] << 4)


def unpack_fp4(packed: torch.Tensor) -> torch.Tensor:
    lo = packed & 0xF
    hi = packed >> 4
    return torch.stack([lo, hi], dim=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def mx_exponent(amax: torch.Tensor, qmax: float) -> torch.Tensor:
    """ceil(log2(amax / qmax)) computed exactly from the fp32 ratio, clamped to [-127, 127]."""
    r = amax.float() / qmax
    m, e = torch.frexp(r)
    exp = torch.where(m == 0.5, e - 1, e).to(torch.int32)
    exp = torch.where(r < 2.0**-126, torch.full_like(exp, -127), exp)
    return exp.clamp(-127, 127)


def exp2i(e: torch.Tensor) -> torch.Tensor:
    return torch.ldexp(torch.ones_like(e, dtype=torch.float32), e.to(torch.int32))


def to_e4m3(x: torch.Tensor) -> torch.Tensor:
    """f32 -> e4m3fn bytes (round to nearest even, saturating at 448)."""
    return x.float().clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def from_e4m3(b: torch.Tensor) -> torch.Tensor:
    return b.view(torch.float8_e4m3fn).float()


# ------------------------------------------------------------------------------------------------
# MX formats
# ------------------------------------------------------------------------------------------------
def quantize_mxfp4(w: torch.Tensor, search: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """[N, K] -> (packed [N, K/2] uint8, sf chunk-layout uint8). MSE search over exponent shifts -2..+2."""
    w = w.float().cpu()
    N, K = w.shape
    assert K % 32 == 0
    blocks = w.reshape(N, K // 32, 32)
    amax = blocks.abs().amax(-1)
    base = mx_exponent(amax, FP4_MAX)
    best = base.clone()
    if search:
        best_err = torch.full(base.shape, float("inf"))
        for d in (2, 1, 0, -1, -2):  # same order as the kernel: ties keep the larger exponent
            e = (base + d).clamp(-127, 127)
            s = exp2i(e)[..., None]
            dq = e2m1_decode(e2m1_encode(blocks / s)) * s
            err = ((dq - blocks) ** 2).sum(-1)
            take = err < best_err
            best = torch.where(take, e, best)
            best_err = torch.where(take, err, best_err)
    codes = e2m1_encode(blocks / exp2i(best)[..., None]).reshape(N, K)
    return pack_fp4(codes), pack_sf((best + 127).to(torch.uint8))


def quantize_mxfp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[M, K] -> (e4m3 bytes [M, K], sf chunk-layout uint8)."""
    x = x.float().cpu()
    M, K = x.shape
    blocks = x.reshape(M, K // 32, 32)
    e = mx_exponent(blocks.abs().amax(-1), E4M3_MAX)
    q = to_e4m3(blocks / exp2i(e)[..., None]).reshape(M, K)
    return q, pack_sf((e + 127).to(torch.uint8))


def dequant_mx(q: torch.Tensor, sf: torch.Tensor, rows: int, K: int, fp4: bool) -> torch.Tensor:
    q = q.cpu()
    vals = e2m1_decode(unpack_fp4(q)) if fp4 else from_e4m3(q)
    e = unpack_sf(sf, rows, K // 32).to(torch.int32) - 127
    scale = exp2i(e.clamp(min=-126)) * torch.where(e < -126, 0.5, 1.0)
    return (vals.reshape(rows, K // 32, 32) * scale[..., None]).reshape(rows, K)


# ------------------------------------------------------------------------------------------------
# NVFP4
# ------------------------------------------------------------------------------------------------
def nvfp4_global_scale(w: torch.Tensor) -> float:
    """Global scale so that the largest block scale maps to e4m3's max: g = 448 * 6 / amax."""
    amax = float(w.abs().max())
    return (E4M3_MAX * FP4_MAX) / amax if amax > 0 else 1.0


def quantize_nvfp4(w: torch.Tensor, global_scale: float | None = None):
    """[N, K] -> (packed [N, K/2], s16 e4m3 [N, K/16] bytes, g). w = v * s / g."""
    w = w.float().cpu()
    N, K = w.shape
    g = nvfp4_global_scale(w) if global_scale is None else global_scale
    blocks = w.reshape(N, K // 16, 16)
    amax = blocks.abs().amax(-1)
    s_q = to_e4m3(amax / FP4_MAX * g)
    s = from_e4m3(s_q)
    safe = torch.where(s > 0, s, torch.ones_like(s))
    codes = torch.where((s > 0)[..., None], e2m1_encode(blocks * g / safe[..., None]), torch.zeros_like(blocks, dtype=torch.uint8))
    return pack_fp4(codes.reshape(N, K)), s_q, g


def dequant_nvfp4(packed: torch.Tensor, s16: torch.Tensor, g: float) -> torch.Tensor:
    vals = e2m1_decode(unpack_fp4(packed.cpu()))
    N, K = vals.shape
    s = from_e4m3(s16.cpu())
    return (vals.reshape(N, K // 16, 16) * s[..., None] / g).reshape(N, K)


def nvfp4_to_mxfp4(packed: torch.Tensor, s16: torch.Tensor, g: float, search: bool = True):
    """Load-time NVFP4 -> MXFP4 conversion (reference: r9700_vllm/quant/nvfp4.py:78)."""
    w = dequant_nvfp4(packed, s16, g)
    # the kernel multiplies by 1/g in fp32; mirror that rounding
    vals = e2m1_decode(unpack_fp4(packed.cpu()))
    N, K = vals.shape
    s = from_e4m3(s16.cpu())
    w = (vals.reshape(N, K // 16, 16) * s[..., None] * torch.tensor(1.0 / g, dtype=torch.float32)).reshape(N, K)
    return quantize_mxfp4(w, search=search)


# ------------------------------------------------------------------------------------------------
# fp8 weight formats
# ------------------------------------------------------------------------------------------------
def quantize_block_fp8(w: torch.Tensor, block: int = 128):
    """[N, K] -> (e4m3 [N, K], fp32 scales [ceil(N/128), ceil(K/128)]), w = q * s."""
    w = w.float().cpu()
    N, K = w.shape
    nb, kb = math.ceil(N / block), math.ceil(K / block)
    pad = torch.zeros(nb * block, kb * block)
    pad[:N, :K] = w
    t = pad.reshape(nb, block, kb, block)
    amax = t.abs().amax(dim=(1, 3))
    s = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = to_e4m3(t / s[:, None, :, None]).reshape(nb * block, kb * block)[:N, :K]
    return q.contiguous(), s


def dequant_block_fp8(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    vals = from_e4m3(q.cpu())
    N, K = vals.shape
    srep = s.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return vals * srep


def block_fp8_to_mxfp8(q: torch.Tensor, s: torch.Tensor, block: int = 128):
    """Load-time block-128 fp8 -> MXFP8 requantisation (the reference requantises to per-row fp8
    instead, r9700_vllm/linear/fp8_block.py:23; per-32 power-of-two scales lose less)."""
    return quantize_mxfp8(dequant_block_fp8(q, s, block))


def quantize_rows_fp8(x: torch.Tensor):
    """Per-token e4m3 with scale amax/448 (reference: kernels/r9k_moe_mxfp4a8.hip:1745)."""
    x = x.float().cpu()
    amax = x.abs().amax(-1, keepdim=True)
    s = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    return to_e4m3(x / s), s.squeeze(-1)
