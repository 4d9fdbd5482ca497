"""All-or-nothing set-up of the symmetric-memory communicator, on CPU gloo ranks: when one rank cannot
allocate or open its region, every rank drops the fused path and keeps the NCCL/gloo collectives
(reference: comm/r9k_ar.py:422-439). The native calls are stood in for by a fake."""
import os
import socket

import torch


class _FakeOps:
    def __init__(self, fail_alloc: bool):
        self.fail_alloc = fail_alloc
        self.freed, self.closed = [], []

    def symm_alloc(self, n):
        if self.fail_alloc:
            raise RuntimeError("cudaMalloc failed (injected)")
        return 4096

    def symm_ipc_handle(self, p):
        return torch.arange(64, dtype=torch.uint8)

    def symm_open(self, h):
        return 8192

    def symm_close(self, p):
        self.closed.append(p)

    def symm_free(self, p):
        self.freed.append(p)


def _worker(rank, world, port, fail_rank, q):
    import torch.distributed as dist

    from r9700_stack_b200 import _native, knobs
    from r9700_stack_b200.parallel import symm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), R9K_PREFILL_AR="nccl", R9K_LOGITS_AG="nccl")
    knobs.refresh()
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = _FakeOps(fail_alloc=(rank == fail_rank))
    _native.ops = lambda: fake  # stand-in for the kernel library
    try:
        c = symm.SymmComm(256, max_tokens=4, calls_per_step=2, device="cpu")
        t = torch.full((4,), float(rank + 1))
        c.all_reduce_(t)  # the fallback collective still works
        q.put((rank, bool(c.fused), t.tolist(), len(fake.freed) + len(fake.closed)))
    finally:
        dist.destroy_process_group()


def _run(fail_rank):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, fail_rank, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (f, t, n)) for r, f, t, n in (q.get(timeout=120) for _ in ps))
    for p in ps:
        p.join(timeout=60)
    return res


def test_one_rank_failing_disables_fused_everywhere():
    res = _run(fail_rank=1)
    assert [res[r][0] for r in (0, 1)] == [False, False]
    assert res[0][1] == [3.0] * 4 and res[1][1] == [3.0] * 4
    assert res[0][2] >= 1  # rank 0 released what it had set up


def test_all_ranks_ok_keeps_fused():
    res = _run(fail_rank=-1)
    assert [res[r][0] for r in (0, 1)] == [True, True]
