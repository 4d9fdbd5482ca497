"""Host-resident tables: int6 / fp8 row formats (CPU), and the UVA gather kernel vs the CPU decode (GPU)."""
import pytest
import torch

from r9700_stack_b200.ops import hostmem as HM


def test_int6_roundtrip():
    x = torch.randn(5, 160) * 0.05
    q = HM.quantize_int6(x)
    assert q.shape == (5, 130)  # the reference's 130-byte rows at dim 160
    y = HM.dequant_int6(q, 160)
    assert float((x - y).abs().max()) <= float(x.abs().max()) / 31 * 0.51 + 1e-6


def test_fp8_roundtrip():
    x = torch.randn(4, 256)
    y = HM.dequant_fp8(HM.quantize_fp8(x), 256)
    torch.testing.assert_close(y, x, rtol=0.07, atol=1e-3)


def test_ngram_ids_deterministic():
    t = torch.tensor([5, 9, 9, 5, 9, 9])
    a = HM.ngram_ids(t, 2, 1000)
    assert a[1] == a[4] and a[2] == a[5] and a[1] != a[2]
    assert int(a.max()) < 1000 and int(a.min()) >= 0


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,dim", [("int6", 160), ("int6", 256), ("fp8", 256)])
def test_host_gather(fmt, dim):
    tab = HM.HostTable.random(1000, dim, fmt, seed=3)
    ids = torch.tensor([0, 999, 17, -1, 5000, 17, 3], dtype=torch.int64, device="cuda")
    out = torch.empty(ids.numel(), dim, dtype=torch.bfloat16, device="cuda")
    tab.gather(ids, out)
    torch.cuda.synchronize()
    ref = tab.gather_ref(ids)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=1e-2, atol=1e-4)
