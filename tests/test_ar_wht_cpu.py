"""CPU checks of the compressed all-reduce oracle (WHT-64 + 4/6-bit codes)."""
import torch

from r9700_stack_b200.parallel import compress as C


def test_wht_orthonormal():
    x = torch.randn(10, 64)
    y = C.wht64(x)
    assert torch.allclose(C.wht64(y), x, atol=1e-5)
    assert torch.allclose(y.norm(dim=-1), x.norm(dim=-1), rtol=1e-5)
    # against the Sylvester matrix
    H = torch.ones(1, 1)
    while H.shape[0] < 64:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    assert torch.allclose(y, x @ H.T / 8, atol=1e-5)


def test_quant_error_and_wire():
    torch.manual_seed(0)
    x = torch.randn(64 * 256).bfloat16()
    for bits, tol in ((6, 0.03), (4, 0.15)):
        out = C.all_reduce_ref([x], bits)
        rel = (out.float() - x.float()).norm() / x.float().norm()
        assert rel < tol, (bits, rel)
        q, s = C.quantize(x, bits)
        assert int(q.abs().max()) <= (1 << (bits - 1)) - 1
    assert C.wire_bytes(4096, 6) == 64 * 50 and C.wire_bytes(4096, 4) == 64 * 34


def test_reduce_is_rank_order_sum():
    torch.manual_seed(1)
    xs = [torch.randn(640).bfloat16() for _ in range(3)]
    out = C.all_reduce_ref(xs, 6).float()
    exact = sum(x.float() for x in xs)
    assert (out - exact).norm() / exact.norm() < 0.05
    # an outlier stays confined to its own 64-block
    y = torch.zeros(128).bfloat16()
    y[3] = 100.0
    o = C.all_reduce_ref([y], 4).float()
    assert o[64:].abs().max() == 0
