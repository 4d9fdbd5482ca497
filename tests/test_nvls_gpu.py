"""NVLS (NVSwitch multicast) all-reduce and all-gather over every visible GPU, one rank each:
identical results on every rank, the all-reduce within one rounding of the rank-ordered fp32 sum,
the all-gather exact, CUDA-graph replays. Skips where the platform offers no multicast object."""
import os
import queue
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inp(rank, n, it, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(7919 * rank + it)
    return torch.randn(n, generator=g).to(dtype)


def _worker(rank, world, port, q):
    from datetime import timedelta

    import torch.distributed as dist

    from r9700_stack_b200.parallel.nvls import NvlsComm
    from r9700_stack_b200.utils import status

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    res = {"errs": [], "available": None, "digests": []}
    try:
        c = NvlsComm(dev, capacity_bytes=64 << 20)
        res["available"] = c.available
        if c.available:
            for it, n in enumerate([8 * world, 4096 * world, 5120 * 16, 8192 * 5120 // 4]):
                n -= n % (8 * world)
                x = _inp(rank, n, it).to(dev)
                y = x.clone()
                c.all_reduce_(y)
                torch.cuda.synchronize(dev)
                ref = sum(_inp(r, n, it).float() for r in range(world))
                err = (y.float().cpu() - ref).abs().max().item()
                if err > 4e-2 * ref.abs().max().item() + 1e-2:
                    res["errs"].append(f"ar n={n} err={err}")
                res["digests"].append(float(y.float().sum()))
                a = _inp(rank, 4 * 1000 + 4, 100 + it, torch.float32)[: (1004 // 4) * 4].to(dev)
                out = torch.empty(world, a.numel(), dtype=torch.float32, device=dev)
                c.all_gather(a, out)
                torch.cuda.synchronize(dev)
                want = torch.stack([_inp(r, 4 * 1000 + 4, 100 + it, torch.float32)[: a.numel()] for r in range(world)])
                if not torch.equal(out.cpu(), want):
                    res["errs"].append(f"ag it={it}")
            # graph replays of interleaved collectives
            x = _inp(rank, 65536, 99).to(dev)
            y = torch.empty_like(x)
            s = torch.cuda.Stream(dev)
            with torch.cuda.stream(s):
                y.copy_(x)
                c.all_reduce_(y)
                torch.cuda.synchronize(dev)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    y.copy_(x)
                    c.all_reduce_(y)
            for _ in range(20):
                g.replay()
            torch.cuda.synchronize(dev)
            ref = sum(_inp(r, 65536, 99).float() for r in range(world))
            if (y.float().cpu() - ref).abs().max().item() > 4e-2 * ref.abs().max().item() + 1e-2:
                res["errs"].append("graph ar")
            res["digests"].append(float(y.float().sum()))
            del g
        status.check()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    q.put((rank, res))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
def test_nvls_collectives():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res, t0 = {}, time.time()
    while len(res) < world and time.time() - t0 < 300:
        try:
            r, v = q.get(timeout=1)
            res[r] = v
        except queue.Empty:
            dead = [i for i, p in enumerate(ps) if p.exitcode not in (None, 0)]
            assert not dead, f"ranks {dead} exited with an error"
    for p in ps:
        p.join(timeout=60)
    assert len(res) == world
    if not res[0]["available"]:
        pytest.skip("no NVSwitch multicast object on this platform")
    assert all(not v["errs"] for v in res.values()), {r: v["errs"] for r, v in res.items()}
    assert all(v["digests"] == res[0]["digests"] for v in res.values()), "ranks differ"
