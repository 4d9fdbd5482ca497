"""Rank-skew race test of the fused decode all-reduce (LL, pull and push protocols): every rank
replays a captured step of mixed-size all-reduce + RMSNorm calls many times while one rank starts
each replay late by a random amount, and the inputs change every replay, so a rank that reused a
buffer too early, or read a peer's previous data, would produce a wrong row.
Reference counterpart: tests/test_ar_race.py:1-16 (one rank burns GPU time before graph replays of
mixed-size all-reduces, 1500 times)."""
import os
import queue
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

H = 1024
SIZES = [1, 16, 3, 8, 16, 2]  # rows per call (the decode batch varies between captured graphs)
REPLAYS = 300


def _worker(rank, world, port, q, mode):
    import random
    from datetime import timedelta

    import torch.distributed as dist

    from r9700_stack_b200 import knobs
    from r9700_stack_b200.parallel.symm import SymmComm
    from r9700_stack_b200.utils import status

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), R9K_AR_MODE=mode)
    knobs.refresh()
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    errs = []
    graph = None
    comm = SymmComm(H, max_tokens=16, calls_per_step=len(SIZES), device=dev, timeout_s=2.0)
    try:
        w = torch.ones(H, dtype=torch.bfloat16, device=dev)
        xs = [torch.zeros(T, H, dtype=torch.bfloat16, device=dev) for T in SIZES]
        ys = [torch.zeros(T, H, dtype=torch.bfloat16, device=dev) for T in SIZES]
        ridx = torch.arange(H, device=dev).float()

        def fill(i):
            # small integers: every partial and every sum is exact in bf16
            for k, x in enumerate(xs):
                rows = torch.arange(x.shape[0], device=dev).float()[:, None]
                x.copy_(((rank + 1) * ((i + k) % 5 + 1) + rows + (ridx % 7)).bfloat16())

        def expect(i):
            out = []
            for k, T in enumerate(SIZES):
                rows = torch.arange(T, device=dev).float()[:, None]
                tot = sum((r + 1) * ((i + k) % 5 + 1) + rows + (ridx % 7) for r in range(world))
                out.append(tot * torch.rsqrt(tot.pow(2).mean(-1, keepdim=True) + 1e-6))
            return out

        def step():
            comm.step_begin()
            for k, T in enumerate(SIZES):
                if comm.mode == "pull":
                    comm.out_buffer(k, T).copy_(xs[k])
                else:
                    comm.push(xs[k], k)
                comm.ar_rmsnorm(k, T, w, 1e-6, False, y=ys[k])

        s = torch.cuda.Stream(dev)
        with torch.cuda.stream(s):
            fill(0)
            step()
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                step()
        rng = random.Random(rank * 7919)
        dist.barrier()
        with torch.cuda.stream(s):
            for i in range(REPLAYS):
                fill(i)
                if rank == 0 and rng.random() < 0.7:
                    torch.cuda._sleep(rng.randrange(1000, 60000))  # start this replay late
                graph.replay()
                if i % 50 == 49 or i == REPLAYS - 1:
                    torch.cuda.synchronize(dev)
                    for k, (y, e) in enumerate(zip(ys, expect(i))):
                        if not torch.allclose(y.float(), e, rtol=1e-2, atol=1e-2):
                            errs.append(f"{mode} replay {i} call {k}")
        torch.cuda.synchronize(dev)
        status.check()
        dist.barrier()
    finally:
        del graph
        torch.cuda.synchronize(dev)
        comm.close()
        dist.destroy_process_group()
    q.put((rank, errs))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
@pytest.mark.parametrize("mode", ["ll", "pull", "push"])
def test_fused_allreduce_rank_skew(mode):
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in ps:
        p.start()
    res, t0 = {}, time.time()
    while len(res) < world and time.time() - t0 < 300:
        try:
            r, errs = q.get(timeout=1)
            res[r] = errs
        except queue.Empty:
            dead = [i for i, p in enumerate(ps) if p.exitcode not in (None, 0)]
            assert not dead, f"ranks {dead} exited with an error"
    for p in ps:
        p.join(timeout=60)
    assert len(res) == world and all(not v for v in res.values()), res
