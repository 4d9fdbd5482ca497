"""NVLink collectives (one-shot / two-shot all-reduce, all-gather, reduce-scatter) vs the exact
rank-ordered reference, on every visible GPU as one rank each (2+ GPUs), plus the single-rank case
and CUDA-graph replay. Inputs are regenerated from per-rank seeds so each rank checks alone."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(rank, n, it):
    g = torch.Generator().manual_seed(1000 * rank + it)
    return torch.randn(n, generator=g).bfloat16()


def _ref_sum(world, n, it):
    acc = torch.zeros(n, dtype=torch.float32)
    for r in range(world):
        acc += _inputs(r, n, it).float()
    return acc.bfloat16()


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from r9700_stack_b200.parallel.collectives import SymmCollectives
    from r9700_stack_b200.utils import status

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        c = SymmCollectives(f"cuda:{rank}", slot_bytes=4 << 20)
        errs = []
        sizes = [8, 4096 * world, 100_003, 4096 * world * 16]
        for it, n in enumerate(sizes):
            x = _inputs(rank, n, it).cuda()
            y = c.all_reduce_oneshot(x)
            if not torch.equal(y.cpu(), _ref_sum(world, n, it)):
                errs.append(f"oneshot n={n}")
            if n % (world * 4096) == 0:
                y2 = c.all_reduce_twoshot(x)
                if not torch.equal(y2.cpu(), _ref_sum(world, n, it)):
                    errs.append(f"twoshot n={n}")
                seg = c.reduce_scatter(x)
                if not torch.equal(seg.cpu(), _ref_sum(world, n, it).view(world, -1)[rank]):
                    errs.append(f"rs n={n}")
            ag = c.all_gather(x)
            if not torch.equal(ag.cpu(), torch.cat([_inputs(r, n, it) for r in range(world)])):
                errs.append(f"ag n={n}")
        # lossy compressed all-reduce: the oracle over every rank's input, identical on all ranks
        from r9700_stack_b200.parallel import compress as C

        for bits in (4, 6):
            n = 4096 * world * 4 + 64
            x = _inputs(rank, n, 50 + bits).cuda()
            y = c.all_reduce_wht(x, bits)
            ref = C.all_reduce_ref([_inputs(r, n, 50 + bits) for r in range(world)], bits)
            if not torch.equal(y.cpu(), ref):
                errs.append(f"wht{bits}")
        # graph replay of interleaved collectives
        x = _inputs(rank, 65536, 99).cuda()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            c.all_reduce_oneshot(x)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                a = c.all_reduce_oneshot(x)
                b = c.all_gather(x)
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        if not torch.equal(a.cpu(), _ref_sum(world, 65536, 99)):
            errs.append("graph ar")
        status.check()
        del g
        c.close()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
def test_collectives_multi_gpu():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    import queue
    import time

    res, t0 = {}, time.time()
    while len(res) < world and time.time() - t0 < 300:
        try:
            r, errs = q.get(timeout=1)
            res[r] = errs
        except queue.Empty:
            # a rank that died (e.g. a CUDA error) fails the test at once instead of after the timeout
            dead = [i for i, p in enumerate(ps) if p.exitcode not in (None, 0)]
            assert not dead, f"ranks {dead} exited with an error"
    for p in ps:
        p.join(timeout=120)
    assert len(res) == world and all(not v for v in res.values()), res


def test_collectives_single_rank():
    from r9700_stack_b200.parallel.collectives import SymmCollectives
    from r9700_stack_b200.utils import status

    c = SymmCollectives("cuda", slot_bytes=1 << 20)
    x = torch.randn(50_000, device="cuda").bfloat16()
    assert torch.equal(c.all_reduce_oneshot(x), x)
    assert torch.equal(c.all_gather(x), x)
    y = torch.randn(4096 * 4, device="cuda").bfloat16()
    assert torch.equal(c.all_reduce_twoshot(y), y)
    torch.cuda.synchronize()
    status.check()
    c.close()
