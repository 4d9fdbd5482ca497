"""Compressed all-reduce kernel (WHT-64 + 4/6-bit codes over the symmetric region) against the
torch oracle, bit for bit: one rank, several ranks emulated on one GPU (publish phase of every
rank first, then the reduce phase of every rank, so every wait is already satisfied), and CUDA
graph replay. The multi-GPU run is in test_collectives_gpu.py."""
import pytest
import torch

from r9700_stack_b200 import _native
from r9700_stack_b200.parallel import compress as C
from r9700_stack_b200.parallel.collectives import SymmCollectives
from r9700_stack_b200.utils import status

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [4, 6])
@pytest.mark.parametrize("n", [64, 4096, 4096 * 3 + 64 * 5])
def test_single_rank(bits, n):
    c = SymmCollectives("cuda", slot_bytes=1 << 20)
    x = (torch.randn(n, device="cuda") * 3).bfloat16()
    y = c.all_reduce_wht(x, bits)
    torch.cuda.synchronize()
    status.check()
    assert torch.equal(y.cpu(), C.all_reduce_ref([x.cpu()], bits))
    c.close()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("bits", [4, 6])
def test_emulated_ranks(world, bits):
    cs = [SymmCollectives("cuda", slot_bytes=1 << 20) for _ in range(world)]
    peers = torch.tensor([c.local_ptr for c in cs], dtype=torch.int64)
    n = 4096 * 5 + 64 * 3
    xs = [torch.randn(n, device="cuda").bfloat16() for _ in range(world)]
    outs = [torch.empty_like(x) for x in xs]
    ops = _native.ops()
    for it in range(3):  # several calls: buffers alternate, epochs advance
        for phase in (1, 2):
            for r, c in enumerate(cs):
                ops.symm_ar_wht(xs[r], outs[r], peers, r, world, c.slot_bytes, c.seq, status.status(c.device), 1.0,
                                bits, phase)
        torch.cuda.synchronize()
        status.check()
        ref = C.all_reduce_ref([x.cpu() for x in xs], bits)
        for r in range(world):
            assert torch.equal(outs[r].cpu(), ref), (it, r)
        xs = [x.roll(64 * (it + 1)) for x in xs]
    for c in cs:
        c.close()


def test_graph_replay():
    c = SymmCollectives("cuda", slot_bytes=1 << 20)
    x = torch.randn(8192, device="cuda").bfloat16()
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        c.all_reduce_wht(x, 6, out=out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            c.all_reduce_wht(x, 6, out=out)
    for i in range(4):
        x.copy_(torch.randn(8192, device="cuda").bfloat16())
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.cpu(), C.all_reduce_ref([x.cpu()], 6))
    status.check()
    assert int(c.seq[0]) == 5
    del g
    c.close()
