"""EXL3-style trellis: CPU oracle properties, and the CUDA dequant / GEMV / grouped-expert GEMV against it."""
import pytest
import torch

from r9700_stack_b200.quant import exl3 as E


def test_oracle_states_wrap():
    # a tile of K=2: 32 words; weight 0's window wraps to the end of the stream
    w = torch.zeros(32, dtype=torch.int16).numpy().view("uint16")
    w[-1] = 0xABCD
    st = E.tile_states(w, 2)
    assert st[0] == (0xABCD << 2) & 0xFFFF  # last 14 bits of the stream, then 2 zero bits
    w2 = w.copy(); w2[:] = 0; w2[0] = 0x8000
    st2 = E.tile_states(w2, 2)
    assert st2[0] == 0x2 and st2[1] == 0x8 and st2[7] == 0x8000 and st2[8] == 0


def test_oracle_rotation_consistent():
    tr, suh, svh = E.random_pack(256, 256, 3, seed=2)
    x = torch.randn(3, 256)
    for cb in (E.MCG, E.MUL1):
        W = E.dequant(tr, suh, svh, 3, cb)
        torch.testing.assert_close(x @ W, E.linear_ref(x, tr, suh, svh, 3, cb), rtol=1e-4, atol=1e-5)
        v = E.decode_tiles(tr, 3, cb).float()
        assert 0.8 < float(v.std()) < 1.5 and abs(float(v.mean())) < 0.1


@pytest.mark.gpu
@pytest.mark.parametrize("K,cb", [(3, E.MCG), (2, E.MUL1), (4, E.MCG), (5, E.MUL1)])
def test_dequant_kernel(K, cb):
    from r9700_stack_b200.ops.exl3 import Exl3Linear

    tr, suh, svh = E.random_pack(256, 384, K, seed=K)
    lin = Exl3Linear(tr.cuda(), suh.cuda(), svh.cuda(), K, cb)
    W = lin.dequant_bf16().w.float().cpu()  # [out, in]
    ref = E.dequant(tr, suh, svh, K, cb).t()
    torch.testing.assert_close(W, ref, rtol=1e-2, atol=1e-2 * float(ref.abs().max()))


@pytest.mark.gpu
@pytest.mark.parametrize("M,n_in,n_out", [(1, 512, 256), (5, 1024, 384), (16, 2048, 256)])
def test_gemv(M, n_in, n_out):
    from r9700_stack_b200.ops.exl3 import Exl3Linear
    from r9700_stack_b200.utils import status

    tr, suh, svh = E.random_pack(n_in, n_out, 3, seed=M)
    lin = Exl3Linear(tr.cuda(), suh.cuda(), svh.cuda(), 3, E.MCG)
    x = torch.randn(M, n_in).bfloat16()
    out = torch.empty(M, n_out, dtype=torch.float32, device="cuda")
    lin.gemv(x.cuda(), out)
    torch.cuda.synchronize()
    status.check()
    ref = E.linear_ref(x.float(), tr, suh, svh, 3, E.MCG)
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-3, atol=1e-3 * float(ref.abs().max()))


@pytest.mark.gpu
def test_grouped_experts_swiglu():
    from r9700_stack_b200.ops.exl3 import random_linear
    from r9700_stack_b200.utils import status

    Ex, H, I = 4, 512, 256
    g = random_linear(H, I, 3, "cuda", seed=1, experts=Ex)
    u = random_linear(H, I, 3, "cuda", seed=2, experts=Ex)
    rows = torch.randn(20, H).bfloat16().cuda()
    work = torch.tensor([[2, 0, 5], [0, 5, 11], [3, 16, 4], [1, 0, 0]], dtype=torch.int32, device="cuda")
    wc = torch.tensor([3], dtype=torch.int32, device="cuda")
    out = torch.zeros(20, I, dtype=torch.bfloat16, device="cuda")
    g.gemv(rows, out, work=work, work_count=wc, n_items=4, rows=16, up=u)
    torch.cuda.synchronize()
    status.check()
    for e, r0, n in [(2, 0, 5), (0, 5, 11), (3, 16, 4)]:
        x = rows[r0:r0 + n].float().cpu()
        a = E.linear_ref(x, g.trellis[e].cpu(), g.suh[e].cpu(), g.svh[e].cpu(), 3, E.MCG)
        b = E.linear_ref(x, u.trellis[e].cpu(), u.suh[e].cpu(), u.svh[e].cpu(), 3, E.MCG)
        ref = torch.nn.functional.silu(a) * b
        got = out[r0:r0 + n].float().cpu()
        torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2 * float(ref.abs().max()))
