"""mHC seam: the PyTorch restatement vs vLLM's torch reference (CPU) and the CUDA seam vs both (GPU)."""
import pytest
import torch

from r9700_stack_b200.ops.mhc import MHCParams, seam_ref


def _params(H, dev="cpu", seed=0):
    g = torch.Generator().manual_seed(seed)
    fn = (torch.randn(24, 4 * H, generator=g) * 0.02).to(dev)
    return MHCParams(fn=fn, scale=torch.tensor([0.8, 1.1, 0.9]).to(dev), base=(torch.randn(24, generator=g) * 0.1).to(dev))


def _inputs(T, H, dev="cpu", seed=1):
    g = torch.Generator().manual_seed(seed)
    R = torch.randn(T, 4, H, generator=g).bfloat16().to(dev)
    so = torch.randn(T, H, generator=g).bfloat16().to(dev)
    post = torch.rand(T, 4, generator=g).to(dev) * 2
    comb = torch.softmax(torch.randn(T, 4, 4, generator=g), -1).to(dev)
    return R, so, post, comb


def test_ref_matches_vllm_torch():
    mt = pytest.importorskip("vllm.model_executor.kernels.mhc.torch")
    H, T = 256, 3
    p = _params(H)
    R, so, post, comb = _inputs(T, H)
    R2, post2, comb2, li = seam_ref(R, p, so, post, comb)
    Rv = mt.mhc_post_torch(so, R, post[..., None], comb)
    assert torch.equal(R2, Rv)
    pv, cv, lv = mt.mhc_pre_torch(Rv, p.fn, p.scale, p.base, p.rms_eps, p.pre_eps, p.sk_eps, p.post_mult, p.sk_repeat)
    torch.testing.assert_close(post2, pv.view(T, 4), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(comb2, cv, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(li.float(), lv.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,fold", [(1, 7168, True), (5, 1024, True), (11, 512, False)])
def test_seam_kernel(T, H, fold):
    from r9700_stack_b200.ops.mhc import seam
    from r9700_stack_b200.utils import status

    p = _params(H, "cuda")
    R, so, post, comb = _inputs(T, H, "cuda")
    args = (so, post, comb) if fold else (None, None, None)
    Rr, pr, cr, lr = seam_ref(R, p, *args)
    R_out = torch.empty_like(R)
    Rk, pk, ck, lk = seam(R, p, *args, R_out=R_out)
    torch.cuda.synchronize()
    status.check()
    # the new streams: one bf16 rounding of an fp32 fma chain (torch's einsum may differ by one ulp)
    d = (Rk.float() - Rr.float()).abs()
    assert float((d > 0).float().mean()) < 0.01 and float(d.max()) <= float(Rr.float().abs().max()) * 2 ** -7
    torch.testing.assert_close(pk, pr, rtol=2e-5, atol=2e-6)
    torch.testing.assert_close(ck, cr, rtol=2e-5, atol=2e-6)
    torch.testing.assert_close(lk.float(), lr.float(), rtol=1e-2, atol=1e-2)
    # in place (R_out aliases R) gives the same result
    R2 = R.clone()
    seam(R2, p, *args)
    torch.cuda.synchronize()
    assert torch.equal(R2, Rk)
