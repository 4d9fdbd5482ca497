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


def fused_decode(a, rank: int, world: int, dev) -> None:
    """The decode all-reduce as the model runs it: per call a producer writes this rank's bf16 partial
    [T, H] (a plain copy standing in for the row-parallel GEMM), then the fused all-reduce + residual +
    RMSNorm + MXFP8 kernel. One step = --calls calls, captured in a CUDA graph; per-call cost = (step
    with the fused kernels - step with the producers only) / calls, max over ranks."""
    from .. import knobs
    from ..ops import linear as L
    from ..parallel.symm import SymmComm
    from ..utils import status

    H, calls = a.hidden, a.calls
    rows = []
    for T in [int(t) for t in a.tokens.split(",")]:
        comm = SymmComm(H, max_tokens=T, calls_per_step=calls, device=dev)
        g = torch.Generator(device=dev).manual_seed(rank)
        part = torch.randn(T, H, generator=g, device=dev).bfloat16()
        resid = torch.randn(T, H, device=dev).bfloat16()
        w = torch.ones(H, device=dev).bfloat16()
        act = L.alloc_act(T, H, dev)

        def step(with_ar: bool):
            comm.step_begin()
            for k in range(calls):
                dst = comm.out_buffer(k, T) if comm.mode == "pull" else None
                if comm.mode == "pull":
                    dst.copy_(part)
                else:
                    comm.push(part, k)
                if with_ar:
                    comm.ar_rmsnorm(k, T, w, 1e-6, True, residual=resid, residual_out=None, quant_out=act)

        res = {"T": T, "H": H, "bytes": T * H * 2, "mode": comm.mode}
        for with_ar in (False, True):
            if comm.mode != "pull" and not with_ar:
                continue
            s = torch.cuda.Stream(dev)
            with torch.cuda.stream(s):
                for _ in range(a.warmup):
                    step(with_ar)
                torch.cuda.synchronize(dev)
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=s):
                    for _ in range(a.reps):
                        step(with_ar)
                gr.replay()
                torch.cuda.synchronize(dev)
                dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                gr.replay()
                e1.record(s)
                torch.cuda.synchronize(dev)
            t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (a.reps * calls)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res["us_per_call_with_ar" if with_ar else "us_per_call_producer"] = round(float(t), 2)
            del gr
        if "us_per_call_producer" in res:
            res["ar_us"] = round(res["us_per_call_with_ar"] - res["us_per_call_producer"], 2)
        status.check()
        torch.cuda.synchronize(dev)
        comm.barrier()
        comm.close()
        rows.append(res)
    if rank == 0:
        for r in rows:
            print(json.dumps({"world": world, "fused_decode": r} | {"knobs": knobs.all_knobs().get("R9K_AR_MODE")}))


def latency(a, rank: int, world: int, dev) -> None:
    """NVLink protocol floor between rank 0 and every other rank: flag ping-pong round trip with
    release/acquire, relaxed, and fenced-relaxed accesses, and the dependent remote load round trip."""
    from .. import _native
    from ..parallel.symm import SymmComm
    from ..utils import status

    comm = SymmComm(128, max_tokens=1, calls_per_step=2, device=dev)
    ops = _native.ops()
    off = 48 * 1024  # unused words of the flag page
    res = {}
    for peer in range(1, world):
        for kind, mode, name in ((0, 0, "pingpong_release_acquire"), (0, 1, "pingpong_relaxed"),
                                 (0, 2, "pingpong_fence_sc"), (1, 1, "remote_load")):
            torch.cuda.synchronize(dev)
            ops.symm_view(comm.local_ptr, off, 1, 64, dev.index or 0).zero_()
            torch.cuda.synchronize(dev)
            dist.barrier()
            if rank in (0, peer):
                other = peer if rank == 0 else 0
                if kind == 1 and rank != 0:
                    t = torch.zeros(2, dtype=torch.int64, device=dev)
                else:
                    t = ops.p2p_probe(comm.peers, rank, other, off, kind, mode, a.iters, status.status(dev), 2.0)
                torch.cuda.synchronize(dev)
                if rank == 0:
                    res.setdefault(f"peer{peer}", {})[name + "_ns"] = round(float(t[0]) / a.iters, 1)
            dist.barrier()
    status.check()
    comm.close()
    if rank == 0:
        print(json.dumps({"world": world, "latency": res}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-kb", default="256,1024,4096,21504")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--fused", action="store_true", help="time the fused decode all-reduce + RMSNorm path")
    ap.add_argument("--tokens", default="1,16")
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--calls", type=int, default=64)
    ap.add_argument("--latency", action="store_true", help="NVLink flag / load round-trip probes")
    ap.add_argument("--iters", type=int, default=2000)
    a = ap.parse_args()
    if a.fused or a.latency:
        rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
        try:
            (latency if a.latency else fused_decode)(a, rank, world, dev)
        finally:
            dist.destroy_process_group()
        return

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
