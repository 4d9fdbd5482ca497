"""CPU oracle tests for the quantisation formats (BASELINE config 1 numerics)."""
import math

import torch

from r9700_stack_b200.quant import formats as F


def test_e2m1_roundtrip_grid():
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    for s in (1.0, -1.0):
        codes = F.e2m1_encode(vals * s)
        assert torch.equal(F.e2m1_decode(codes), vals * s if s > 0 else torch.where(vals == 0, vals, -vals))


def test_e2m1_ties_to_even():
    x = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 100.0])
    expect = torch.tensor([0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0])
    assert torch.equal(F.e2m1_decode(F.e2m1_encode(x)), expect)


def test_pack_unpack_fp4():
    codes = torch.randint(0, 16, (7, 64), dtype=torch.uint8)
    assert torch.equal(F.unpack_fp4(F.pack_fp4(codes)), codes)


def test_mx_exponent_exact():
    amax = torch.tensor([6.0, 6.0001, 3.0, 12.0, 0.0, 448.0, 449.0])
    e = F.mx_exponent(amax, 6.0)
    assert e.tolist()[:4] == [0, 1, -1, 1]
    assert e[4] == -127
    e8 = F.mx_exponent(amax[5:], 448.0)
    assert e8.tolist() == [0, 1]


def test_sf_layout_is_a_permutation():
    rows, kb = 256, 16
    off = F.sf_offsets(rows, kb).reshape(-1)
    assert off.unique().numel() == rows * kb
    assert int(off.max()) < F.sf_num_bytes(rows, kb)
    # row 33, kblock 5 -> chunk 1, byte (1*16 + 1*4 + 1)
    assert int(F.sf_offsets(rows, kb)[33, 5]) == 512 + 1 * 16 + 1 * 4 + 1


def test_mxfp4_error_bounded_and_search_helps():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(256, 512, generator=g) * 0.02
    q0, s0 = F.quantize_mxfp4(w, search=False)
    q1, s1 = F.quantize_mxfp4(w, search=True)
    d0 = F.dequant_mx(q0, s0, 256, 512, fp4=True)
    d1 = F.dequant_mx(q1, s1, 256, 512, fp4=True)
    e0 = ((d0 - w) ** 2).sum()
    e1 = ((d1 - w) ** 2).sum()
    assert e1 <= e0
    rel = math.sqrt(float(e1 / (w**2).sum()))
    assert rel < 0.12


def test_mxfp8_roundtrip():
    x = torch.randn(40, 256)
    q, s = F.quantize_mxfp8(x)
    d = F.dequant_mx(q, s, 40, 256, fp4=False)
    assert float((d - x).abs().max() / x.abs().max()) < 0.07


def test_nvfp4_to_mxfp4_config1():
    """4096x4096 N(0, 0.02) -> NVFP4 -> MXFP4 (+-2 search); Y = X W^T vs fp32."""
    g = torch.Generator().manual_seed(0)
    K = 4096
    w = torch.randn(K, K, generator=g) * 0.02
    x = torch.randn(16, K, generator=g).bfloat16().float()
    packed, s16, gs = F.quantize_nvfp4(w)
    w_nv = F.dequant_nvfp4(packed, s16, gs)
    pm, sm = F.nvfp4_to_mxfp4(packed, s16, gs, search=True)
    w_mx = F.dequant_mx(pm, sm, K, K, fp4=True)
    y_ref = x @ w.T
    y_nv = x @ w_nv.T
    y_mx = x @ w_mx.T
    rel_nv = float((y_nv - y_ref).norm() / y_ref.norm())
    rel_mx = float((y_mx - y_ref).norm() / y_ref.norm())
    assert rel_nv < 0.12 and rel_mx < 0.15
    # block-fp8 path with per-token fp8 activations
    qb, sb = F.quantize_block_fp8(w)
    xq, xs = F.quantize_rows_fp8(x)
    y_fp8 = (F.from_e4m3(xq) * xs[:, None]) @ F.dequant_block_fp8(qb, sb).T
    assert float((y_fp8 - y_ref).norm() / y_ref.norm()) < 0.05
