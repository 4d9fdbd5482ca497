"""All-reduce micro-benchmark over the ranks of one node: exact one-shot / two-shot NVLink kernels,
the lossy WHT-64 4/6-bit compressed kernel and NCCL, per message size. Each candidate is captured
into a CUDA graph of ``--reps`` calls and replayed; the time is CUDA-event device time, the MAX over
ranks. Bus bandwidth uses NCCL's convention for all-reduce (2 (W-1)/W x bytes / time).

    timeout -k 60 300 torchrun --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29511 \\
        -m r9700_stack_b200.tuning.arbench --sizes-kb 1024,4096,21504

The reference's counterpart is its compressed-AR sweep (comm/r9k_ar4.py, tests/test_ar_wht.py
timing sections) and calibration table (comm/calibrate.py).
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-kb", default="256,1024,4096,21504")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()

    from ..parallel.collectives import SymmCollectives
    from ..utils import status

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    sizes = [int(s) * 1024 for s in a.sizes_kb.split(",")]
    c = SymmCollectives(dev, slot_bytes=max(max(sizes), world * max(sizes) * 50 // 128) + (1 << 20))
    rows = []
    graphs = []
    try:
        for nbytes in sizes:
            n = nbytes // 2
            n -= n % (world * 4096)
            x = torch.randn(n, device=dev).bfloat16()
            out = torch.empty_like(x)
            cands = {
                "oneshot": lambda: c.all_reduce_oneshot(x, out),
                "twoshot": lambda: c.all_reduce_twoshot(x, out),
                "wht6": lambda: c.all_reduce_wht(x, 6, out),
                "wht4": lambda: c.all_reduce_wht(x, 4, out),
                "nccl": lambda: dist.all_reduce(out),
            }
            res = {"bytes": n * 2}
            for name, fn in cands.items():
                s = torch.cuda.Stream(dev)
                with torch.cuda.stream(s):
                    for _ in range(a.warmup):
                        fn()
                    torch.cuda.synchronize(dev)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=s):
                        for _ in range(a.reps):
                            fn()
                    graphs.append(g)
                    g.replay()
                    torch.cuda.synchronize(dev)
                    dist.barrier()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(s)
                    g.replay()
                    e1.record(s)
                    torch.cuda.synchronize(dev)
                t = torch.tensor([e0.elapsed_time(e1) / a.reps], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                us = float(t) * 1e3
                res[name] = {"us": round(us, 1), "busbw_gbs": round(2 * (world - 1) / world * n * 2 / (us * 1e-6) / 1e9, 1)}
            rows.append(res)
        status.check()
        if rank == 0:
            for r in rows:
                print(json.dumps({"world": world} | r))
    finally:
        g = None
        graphs.clear()  # graphs holding NCCL calls go before the process group
        torch.cuda.synchronize(dev)
        c.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
