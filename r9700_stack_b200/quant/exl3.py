"""EXL3-style trellis weights: format, CPU oracle and synthetic packs.

A quantised linear [in -> out] is stored as
  * ``trellis`` int16 [in/16, out/16, 16*K]: one tile per 16 inputs x 16 outputs, 256 weights coded
    in 256*K bits (K = bits per weight, 1..8);
  * ``suh`` f16 [in]:  input-side sign/scale vector, applied before the input rotation;
  * ``svh`` f16 [out]: output-side sign/scale vector, applied after the output rotation;
  * the codebook: ``mcg`` or ``mul1``.
(the tensor set and codebook names of exllamav3's format, as the reference describes it:
notes/exl3-plan.md "The checkpoint", r9700_vllm/quant/exl3.py:5-15.)

Decode of one tile (this module is the definition the CUDA kernels are tested against):
  * the tile's 16K words form a circular bitstream of 256K bits, word w's bit 15 first;
  * weight i (0..255) reads the 16-bit window ending at bit (i + 1) K (wrapping around), i.e. its K
    new bits in the low bits of a state that overlaps its predecessors' (a tail-biting trellis);
  * ``mcg``:  x = state * 0xCBAC1FED mod 2^32; x = (x & 0x8FFF8FFF) ^ 0x3B603B60;
              value = fp16(low half of x) + fp16(high half of x), rounded to fp16;
    ``mul1``: x = state * 0x83DCD12D mod 2^32; s = sum of the 4 bytes of x;
              value = fp16 fma((1024 + s), fp16 0x1EEE, fp16 0xC931) (one rounding);
    these are the codebook hash constants of the format;
  * weight i sits at tile row i // 16 (input) and column i % 16 (output) -- this layout is ours; a
    pack written by exllamav3 orders weights inside a tile for its own MMA fragments and would need a
    re-layout at load, which is not implemented here.
The linear then computes y = had_out(had_in(x * suh) @ W') * svh, where had is the 128-point
Walsh-Hadamard transform (Sylvester order, scaled by 1/sqrt(128)) over consecutive 128-blocks.
"""
from __future__ import annotations

import math

import numpy as np
import torch

MCG, MUL1 = 1, 2
_MCG_MUL, _MUL1_MUL = 0xCBAC1FED, 0x83DCD12D


def _h(bits: np.ndarray) -> np.ndarray:
    return bits.astype(np.uint16).view(np.float16).astype(np.float64)


def codebook(state: np.ndarray, cb: int) -> np.ndarray:
    """16-bit states -> fp16 values (numpy)."""
    s = state.astype(np.uint64)
    if cb == MCG:
        x = (s * _MCG_MUL) & 0xFFFFFFFF
        x = (x & 0x8FFF8FFF) ^ 0x3B603B60
        v = _h(x & 0xFFFF) + _h(x >> 16)
    else:
        x = (s * _MUL1_MUL) & 0xFFFFFFFF
        sb = (x & 0xFF) + ((x >> 8) & 0xFF) + ((x >> 16) & 0xFF) + ((x >> 24) & 0xFF)
        v = (1024.0 + sb.astype(np.float64)) * _h(np.array(0x1EEE)) + _h(np.array(0xC931))
    return v.astype(np.float16)


def tile_states(words: np.ndarray, K: int) -> np.ndarray:
    """words [16K] uint16 -> [256] 16-bit states."""
    nb = 256 * K
    bits = np.unpackbits(words.astype(">u2").view(np.uint8))  # MSB first per word
    assert bits.size == nb
    ends = (np.arange(256) + 1) * K
    idx = (ends[:, None] - 16 + np.arange(16)[None, :]) % nb
    w = bits[idx].astype(np.uint32)
    return (w * (1 << np.arange(15, -1, -1, dtype=np.uint32))[None, :]).sum(1).astype(np.uint32)


def decode_tiles(trellis: torch.Tensor, K: int, cb: int) -> torch.Tensor:
    """trellis int16 [in/16, out/16, 16K] -> W' fp16 [in, out] (before rotations)."""
    t = trellis.cpu().numpy().view(np.uint16)
    ti, to, L = t.shape
    assert L == 16 * K
    out = np.zeros((ti * 16, to * 16), dtype=np.float16)
    for a in range(ti):
        for b in range(to):
            v = codebook(tile_states(t[a, b], K), cb).reshape(16, 16)
            out[16 * a:16 * a + 16, 16 * b:16 * b + 16] = v
    return torch.from_numpy(out)


def hadamard_matrix(n: int = 128) -> torch.Tensor:
    """Sylvester-order Hadamard matrix H_n (entries +-1): H_2n = [[H, H], [H, -H]]."""
    H = torch.ones(1, 1)
    while H.shape[0] < n:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    return H


_H128 = None


def had128(x: torch.Tensor) -> torch.Tensor:
    """Normalised 128-point Walsh-Hadamard transform along the last dim (in 128-blocks)."""
    global _H128
    if _H128 is None:
        _H128 = hadamard_matrix(128).double()
    n = x.shape[-1]
    assert n % 128 == 0
    y = x.double().reshape(*x.shape[:-1], n // 128, 128) @ _H128.to(x.device)
    return (y / math.sqrt(128.0)).reshape(x.shape).to(x.dtype)


def dequant(trellis, suh, svh, K: int, cb: int) -> torch.Tensor:
    """Effective weight W [in, out] fp32 with y = x @ W (rotations folded in)."""
    Wp = decode_tiles(trellis, K, cb).float()
    # y = had(had(x * suh) @ W') * svh  ->  W = diag(suh) Hin W' Hout diag(svh) (had is symmetric)
    W = had128(Wp.t()).t()  # Hin @ W'  (columns transformed along the input dim)
    W = had128(W)  # @ Hout (rows transformed along the output dim)
    return suh.float().cpu()[:, None] * W * svh.float().cpu()[None, :]


def linear_ref(x: torch.Tensor, trellis, suh, svh, K: int, cb: int) -> torch.Tensor:
    xr = had128(x.float().cpu() * suh.float().cpu())
    y = xr @ decode_tiles(trellis, K, cb).float()
    return had128(y) * svh.float().cpu()


def random_pack(n_in: int, n_out: int, K: int, seed: int = 0, scale: float = 0.02):
    """Synthetic pack: uniform random trellis words (every word pattern is a valid code), random input
    signs, per-output scales ~ U(0.5, 1.5) x scale with random signs."""
    g = torch.Generator().manual_seed(seed)
    tr = torch.randint(-32768, 32768, (n_in // 16, n_out // 16, 16 * K), generator=g, dtype=torch.int32).to(torch.int16)
    suh = (torch.randint(0, 2, (n_in,), generator=g) * 2 - 1).to(torch.float16)
    sv = (torch.rand(n_out, generator=g) + 0.5) * scale
    svh = (sv * (torch.randint(0, 2, (n_out,), generator=g) * 2 - 1)).to(torch.float16)
    return tr, suh, svh
