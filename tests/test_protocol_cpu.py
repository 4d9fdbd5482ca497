"""CPU-rank tests of the collectives' pull protocol (epochs, double buffering, bounded waits):
several processes with random scheduling skew run many all-reduces over shared-memory regions;
a rank that stops publishing makes the others fail with a timeout instead of hanging."""
import random
import time

import torch
import torch.multiprocessing as mp

from r9700_stack_b200.parallel.protocol_sim import ProtocolTimeout, SimRank, SimRegions


def _worker(rank, world, regions, iters, n, stop_at, results, start):
    rng = random.Random(rank)
    sr = SimRank(regions, rank, world, timeout_s=1.0)
    start.wait(timeout=120)  # spawned ranks finish importing at different times; the skew under test starts here
    try:
        for it in range(iters):
            if stop_at is not None and rank == world - 1 and it == stop_at:
                return  # this rank leaves between calls
            if rng.random() < 0.3:
                time.sleep(rng.random() * 0.003)
            x = torch.full((n,), float(rank + 1) * (it + 1), dtype=torch.float64)
            out = sr.all_reduce(x)
            expect = sum(float(r + 1) for r in range(world)) * (it + 1)
            if not torch.all(out == expect):
                results[rank] = f"wrong at {it}"
                return
        results[rank] = "ok"
    except ProtocolTimeout as e:
        results[rank] = f"timeout: {e}"


def _run(world, iters, stop_at=None):
    ctx = mp.get_context("spawn")
    regions = SimRegions(world, 64)
    mgr = ctx.Manager()
    results = mgr.dict()
    start = ctx.Barrier(world)
    ps = [ctx.Process(target=_worker, args=(r, world, regions, iters, 64, stop_at, results, start))
          for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return dict(results)


def test_skewed_ranks_agree():
    res = _run(3, 150)
    assert all(v == "ok" for v in res.values()), res


def test_dropped_rank_times_out():
    res = _run(3, 20, stop_at=5)
    assert all(res[r].startswith("timeout") for r in (0, 1)), res
