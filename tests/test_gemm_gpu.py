"""tcgen05 GEMM core and quantisation kernels vs the fp32 CPU oracle (sm_100a)."""
import pytest
import torch

from r9700_stack_b200.quant import formats as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from r9700_stack_b200.ops import linear

    return linear


def _check_status():
    from r9700_stack_b200.utils import status

    torch.cuda.synchronize()
    status.check()


def test_quant_weight_mxfp4_matches_oracle(L):
    torch.manual_seed(0)
    w = torch.randn(256, 512) * 0.02
    mw = L.mx_from_float(w.cuda(), fp4=True, search=True)
    q, s = F.quantize_mxfp4(w, search=True)
    assert torch.equal(mw.q.cpu(), q)
    assert torch.equal(mw.sf.cpu(), s)
    torch.testing.assert_close(mw.dequant().cpu(), F.dequant_mx(q, s, 256, 512, True))


def test_quant_act_mxfp8_matches_oracle(L):
    torch.manual_seed(1)
    x = torch.randn(37, 512).bfloat16()
    a = L.quant_act(x.cuda())
    q, s = F.quantize_mxfp8(x.float())
    assert torch.equal(a.q.cpu(), q)
    assert torch.equal(a.sf.cpu()[: s.numel()], s)


def test_nvfp4_to_mxfp4_matches_oracle(L):
    torch.manual_seed(2)
    w = torch.randn(128, 256) * 0.02
    packed, s16, g = F.quantize_nvfp4(w)
    pk_d, s16_d, g_d = L.nvfp4_quantize(w.cuda(), global_scale=g)
    assert torch.equal(pk_d.cpu(), packed) and torch.equal(s16_d.cpu(), s16)
    mw = L.mx_from_nvfp4(pk_d, s16_d, g, search=True)
    pm, sm = F.nvfp4_to_mxfp4(packed, s16, g, search=True)
    assert torch.equal(mw.q.cpu(), pm)
    assert torch.equal(mw.sf.cpu(), sm)


def test_rmsnorm_quant(L):
    torch.manual_seed(3)
    M, K = 9, 1024
    x = torch.randn(M, K).bfloat16().cuda()
    r = torch.randn(M, K).bfloat16().cuda()
    w = (torch.randn(K) * 0.1).bfloat16().cuda()
    y = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    r_out = torch.empty_like(r)
    act = L.alloc_act(M, K, "cuda")
    L.rmsnorm(x, w, 1e-6, plus_one=True, residual=r, residual_out=r_out, out=y, quant_out=act)
    h = (x.float() + r.float()).bfloat16().float()
    ref = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + w.float())
    torch.testing.assert_close(r_out.float(), h)
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=1e-2)
    q, s = F.quantize_mxfp8(y.float().cpu())
    assert torch.equal(act.q.cpu(), q)
    assert torch.equal(act.sf.cpu()[: s.numel()], s)


def _ref_gemm(x_act, w_dq):
    return x_act @ w_dq.T


@pytest.mark.parametrize("fp4", [True, False])
@pytest.mark.parametrize("N,K,M", [(128, 128, 1), (256, 512, 16), (384, 1024, 40), (200, 512, 7), (256, 512, 130),
                                   (128, 4096, 1), (640, 2048, 300), (5120, 4096, 16), (640, 256, 5), (128, 8192, 3),
                                   (2048, 512, 64), (1152, 17408, 2), (2060, 1024, 513), (384, 512, 256)])
def test_gemm_mx(L, fp4, N, K, M):
    torch.manual_seed(N + K + M)
    w = torch.randn(N, K) * 0.02
    x = torch.randn(M, K)
    mw = L.mx_from_float(w.cuda(), fp4=fp4)
    xa = L.quant_act(x.bfloat16().cuda())
    w_dq = mw.dequant().cpu()
    x_dq = F.dequant_mx(xa.q.cpu(), xa.sf.cpu(), M, K, fp4=False)
    y = L.mx_linear(xa, mw, out_dtype=torch.float32)
    _check_status()
    ref = _ref_gemm(x_dq, w_dq)
    torch.testing.assert_close(y.cpu(), ref, rtol=1e-3, atol=1e-3 * float(ref.abs().max()))
    # bf16 output + residual
    res = torch.randn(M, N).bfloat16().cuda()
    y2 = L.mx_linear(xa, mw, residual=res)
    _check_status()
    torch.testing.assert_close(y2.float().cpu(), ref + res.float().cpu(), rtol=2e-2, atol=2e-2 * float(ref.abs().max()))


@pytest.mark.parametrize("N,K,M", [(256, 512, 3), (512, 1024, 64), (256, 256, 200), (2048, 4096, 16), (128, 8192, 1)])
def test_gemm_swiglu_mxfp8(L, N, K, M):
    torch.manual_seed(7)
    wg = torch.randn(N, K) * 0.05
    wu = torch.randn(N, K) * 0.05
    x = torch.randn(M, K)
    g = L.mx_from_float(wg.cuda())
    u = L.mx_from_float(wu.cuda())
    xa = L.quant_act(x.bfloat16().cuda())
    h = L.mx_swiglu(xa, g, u)
    _check_status()
    x_dq = F.dequant_mx(xa.q.cpu(), xa.sf.cpu(), M, K, fp4=False)
    gr = x_dq @ g.dequant().cpu().T
    ur = x_dq @ u.dequant().cpu().T
    href = torch.nn.functional.silu(gr) * ur
    hd = F.dequant_mx(h.q.cpu(), h.sf.cpu(), M, N, fp4=False)
    err = (hd - href).abs()
    tol = 0.07 * href.abs().reshape(M, N // 32, 32).amax(-1).repeat_interleave(32, 1) + 1e-6
    assert bool((err <= tol).all()), float((err / tol).max())


def test_swiglu_split_matches_dual(L):
    """Prefill-sized M takes two GEMMs + swiglu_quant_mxfp8; it agrees with the dual-accumulator kernel
    (the only difference is the bf16 rounding of the gate / up outputs before the activation)."""
    torch.manual_seed(9)
    N, K, M = 512, 1024, 300
    g = L.mx_from_float((torch.randn(N, K) * 0.05).cuda())
    u = L.mx_from_float((torch.randn(N, K) * 0.05).cuda())
    xa = L.quant_act(torch.randn(M, K).bfloat16().cuda())
    assert M >= L.SWIGLU_SPLIT_M
    split = L.mx_swiglu(xa, g, u)
    old = L.SWIGLU_SPLIT_M
    L.SWIGLU_SPLIT_M = 1 << 30
    try:
        dual = L.mx_swiglu(xa, g, u)
    finally:
        L.SWIGLU_SPLIT_M = old
    _check_status()
    a = F.dequant_mx(split.q.cpu(), split.sf.cpu(), M, N, fp4=False)
    b = F.dequant_mx(dual.q.cpu(), dual.sf.cpu(), M, N, fp4=False)
    # one e4m3 step at the top of a block is 32/448 of the block's amax; the bf16 rounding of the gate /
    # up outputs may flip a rounding (or the block exponent), never more than about two such steps
    tol = 0.15 * b.abs().reshape(M, N // 32, 32).amax(-1).repeat_interleave(32, 1) + 1e-6
    assert bool(((a - b).abs() <= tol).all())
    assert float(torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0)) > 0.999


@pytest.mark.parametrize("N,K,M", [(128, 64, 1), (256, 512, 16), (384, 1024, 100), (256, 256, 513), (2048, 4096, 8),
                                   (2060, 512, 300)])
def test_gemm_bf16(L, N, K, M):
    torch.manual_seed(11)
    w = (torch.randn(N, K) * 0.05).bfloat16()
    x = torch.randn(M, K).bfloat16()
    y = L.bf16_linear(x.cuda(), L.BF16Weight(w.cuda()), out_dtype=torch.float32)
    _check_status()
    ref = x.float() @ w.float().T
    torch.testing.assert_close(y.cpu(), ref, rtol=1e-3, atol=1e-3 * float(ref.abs().max()))


def test_stream_k_is_deterministic(L):
    torch.manual_seed(21)
    w = L.mx_from_float((torch.randn(3072, 8192) * 0.02).cuda())
    x = L.quant_act(torch.randn(16, 8192).bfloat16().cuda())
    a = L.mx_linear(x, w, out_dtype=torch.float32)
    b = L.mx_linear(x, w, out_dtype=torch.float32)
    _check_status()
    assert torch.equal(a, b)


@pytest.mark.parametrize("fp4", [True, False])
@pytest.mark.parametrize("N,K,M", [(200, 512, 7), (5120, 4096, 16), (384, 1024, 300)])
def test_gemm_tiled_weights_match_rowmajor(L, fp4, N, K, M):
    torch.manual_seed(5)
    mw = L.mx_from_float((torch.randn(N, K) * 0.02).cuda(), fp4=fp4)
    mt = mw.to_tiled()
    assert torch.equal(mt.rowmajor_q(), mw.q)
    xa = L.quant_act(torch.randn(M, K).bfloat16().cuda())
    a = L.mx_linear(xa, mw, out_dtype=torch.float32)
    b = L.mx_linear(xa, mt, out_dtype=torch.float32)
    _check_status()
    assert torch.equal(a, b)
    # fused swiglu on tiled weights
    g, u = mw, L.mx_from_float((torch.randn(N, K) * 0.02).cuda(), fp4=fp4)
    if N % 32 == 0:
        h1 = L.mx_swiglu(xa, g, u)
        h2 = L.mx_swiglu(xa, g.to_tiled(), u.to_tiled())
        _check_status()
        assert torch.equal(h1.q, h2.q)
