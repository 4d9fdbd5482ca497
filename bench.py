"""Headline benchmark: decode tok/s (1 and 16 streams) and 8k-prompt prefill tok/s of the dense hybrid
GDN/attention 27B-class model, tensor-parallel over the job's GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W]            # this framework
    python bench.py --impl reference ...                           # the reference (prints unavailable)
    python bench.py --impl vllm ...                                # stock vLLM bf16 on the same shapes

For N > 1 launch with torchrun (one rank per GPU, NCCL). Weights are random N(0, 0.02) quantised to
NVFP4 (converted to MXFP4 at load), lm_head block fp8 (-> MXFP8), fp8 KV cache; prompts are uniform
random token ids. Rank 0 prints one JSON line.

Timing: W untimed decode steps, then exactly K decode steps of 16 streams, each step's CUDA-graph replay
bracketed by CUDA events on the launching stream; a barrier + synchronize on both sides; the max over
ranks. Each step reads all weights (~15 GB at TP=1), far more than L2 (126 MB), so no L2 flush is
needed. The ``e2e`` figure times the same K steps through the public ``LLM.step()`` API (host
scheduling, per-step H2D of the step's metadata from pinned memory, D2H of the sampled tokens).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "decode tok/s (1 and 16 streams), prefill tok/s @8k prompt, device-timed max/rank"
BASELINE_DECODE16 = 640.0  # reference: 27B NVFP4 TP2, 16 streams (README.md:69)
BASELINE_FLASHNEXT16 = 913.0  # reference: Flash-Next MTP-3 TP4, 16 streams (README.md:70)
REF_DIR = os.path.join(HERE, "baseline", "_ref")


def reference_probe() -> str:
    """Try the reference's own stock entry path (installed unmodified under baseline/_ref): its vLLM
    platform plugin ``detect()`` and its kernel library. Returns the observed reason it cannot run."""
    if not os.path.isdir(os.path.join(REF_DIR, "r9700_vllm")):
        return "reference not installed under baseline/_ref"
    sys.path.insert(0, REF_DIR)
    seen = []
    try:
        import r9700_vllm.platform as rp

        got = rp.detect()
        seen.append(f"r9700_vllm.platform.detect() returned {got!r} (it activates only where vLLM's ROCm probe "
                    "finds a ROCm GPU)")
    except Exception as e:  # noqa: BLE001 - the failure is the finding
        seen.append(f"r9700_vllm.platform.detect() raised {type(e).__name__}: {str(e).splitlines()[0][:160]}")
    try:
        import glob

        import r9700_vllm

        libs = glob.glob(os.path.join(os.path.dirname(r9700_vllm.__file__), "**", "libr9k*.so"), recursive=True)
        seen.append("libr9k.so present" if libs else
                    "libr9k.so absent: its 23 .hip kernel sources build only with hipcc for gfx1201 (not in this image)")
    except Exception as e:  # noqa: BLE001
        seen.append(f"import r9700_vllm raised {type(e).__name__}")
    return "reference is a ROCm/gfx1201 vLLM plugin with no CUDA path; observed: " + "; ".join(seen)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "vllm"],
                    help="ours | reference (the installed reference's stock path) | vllm (stock vLLM, bf16, "
                         "NCCL + cuBLAS: a second comparator, see bench_vllm.py)")
    ap.add_argument("--streams", type=int, default=16)
    ap.add_argument("--prompt-len", type=int, default=8192)
    ap.add_argument("--layers", type=int, default=0, help="override layer count (debug only; invalid for the metric)")
    ap.add_argument("--model", default="dense27b", choices=["dense27b", "flashnext"],
                    help="dense27b: BASELINE config 2 (headline); flashnext: config 3 (hybrid MoE)")
    ap.add_argument("--no-prefill-metric", action="store_true")
    ap.add_argument("--diag", action="store_true",
                    help="after the timed steps, print a second JSON line with a per-family step ledger (torch "
                         "profiler) from every rank; diagnostics only, not part of the metric")
    return ap.parse_args()


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons during the timed region: nvidia-smi every 100 ms,
    plus NVML read every 10 ms from a thread (read-only queries), so a region of a few hundred ms still
    holds many samples. Only samples whose timestamp falls inside the marked region are kept (the
    nearest one if the region is shorter than a period)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index="0"):
        self.proc = None
        self.gpu = gpu_index
        import tempfile

        fd, self.path = tempfile.mkstemp(prefix="r9k_clocks_", suffix=".csv")
        os.close(fd)
        self.t0 = self.t1 = None
        self.nvml: list = []
        self._halt = None
        self._thread = None

    def _nvml_loop(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = (pynvml.nvmlDeviceGetHandleByUUID(self.gpu) if str(self.gpu).startswith("GPU-")
                 else pynvml.nvmlDeviceGetHandleByIndex(int(self.gpu)))
            cmax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            bits = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}
            while not self._halt.is_set():
                clk = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                r = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.nvml.append((time.time(), clk, cmax, [n for n, b in bits.items() if r & b]))
                self._halt.wait(0.01)
        except Exception:
            return

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
            deadline = time.time() + 10
            while time.time() < deadline and os.path.getsize(self.path) == 0:
                time.sleep(0.05)
        except Exception:
            self.proc = None
        import threading

        self._halt = threading.Event()
        self._thread = threading.Thread(target=self._nvml_loop, daemon=True)
        self._thread.start()

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self) -> dict:
        if self._halt is not None:
            self._halt.set()
            self._thread.join(timeout=5)
        samples = list(self.nvml)
        if self.proc is None and not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()
        from datetime import datetime

        for line in (open(self.path) if self.proc is not None else []):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 10:
                continue
            try:
                ts = datetime.strptime(p[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clk, cmax = float(p[2]), float(p[3])
            except ValueError:
                continue
            samples.append((ts, clk, cmax, [n for n, v in zip(self.NAMES, p[6:10]) if v.lower() == "active"]))
        try:
            os.unlink(self.path)
        except OSError:
            pass
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        samples.sort(key=lambda x: x[0])
        t0, t1 = self.t0 or samples[0][0], self.t1 or samples[-1][0]
        inside = [x for x in samples if t0 <= x[0] <= t1]
        if not inside:
            mid = 0.5 * (t0 + t1)
            inside = [min(samples, key=lambda x: abs(x[0] - mid))]
        reasons = sorted({r for x in inside for r in x[3]})
        return {
            "sm_mhz": statistics.median(x[1] for x in inside),
            "sm_max_mhz": max(x[2] for x in inside),
            "reasons": reasons,
            "samples": len(inside),
        }


def _smi_id(dev) -> str:
    """nvidia-smi's name for this process's GPU: its UUID (robust to CUDA_VISIBLE_DEVICES)."""
    import torch

    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index or 0)


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": reference_probe(), "metric": METRIC}))
        return 0
    if args.impl == "vllm":
        import bench_vllm

        return bench_vllm.run(args, METRIC)

    import numpy as np
    import torch

    from r9700_stack_b200 import _native
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, ParallelConfig, flashnext_moe, qwen27b_hybrid
    from r9700_stack_b200.parallel.comm import NcclComm, init_distributed

    rank, world, local = init_distributed()
    dev = torch.device("cuda", local)
    cfg = qwen27b_hybrid() if args.model == "dense27b" else flashnext_moe()
    base16 = BASELINE_DECODE16 if args.model == "dense27b" else BASELINE_FLASHNEXT16
    if args.layers:
        cfg = cfg.scaled(layers=args.layers)
    S, P = args.streams, args.prompt_len
    comm = None
    if world > 1 or os.environ.get("R9K_BENCH_SYMM") == "1":
        from r9700_stack_b200.parallel.symm import SymmComm

        # decode all-reduces fused into the row-parallel GEMMs and the following norms (NVLink P2P);
        # prefill-sized messages go through NCCL
        comm = SymmComm(cfg.hidden, max_tokens=S, calls_per_step=2 * cfg.layers, device=dev)
    ec = EngineConfig(max_batch=S, max_model_len=P + args.warmup + 2 * args.steps + 64, max_prefill_tokens=P,
                      cuda_graphs=True, graph_batch_sizes=[1, 2, 4, 8, 16])
    t0 = time.time()
    llm = LLM(cfg, ec, ParallelConfig(tp_size=world, tp_rank=rank), device=dev, seed=0, comm=comm)
    build_s = time.time() - t0

    def barrier_sync():
        torch.cuda.synchronize(dev)
        if comm is not None:
            comm.barrier()
        torch.cuda.synchronize(dev)

    rng = np.random.default_rng(1234)
    prompt = lambda: rng.integers(0, cfg.vocab, P).tolist()

    # ---------------- prefill @8k (1 stream): one warm-up prefill, then two timed ----------------
    prefill_ms = []
    if not args.no_prefill_metric:
        for it in range(3):
            llm.add_request(prompt(), SamplingParams(max_tokens=1))
            barrier_sync()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            llm.step()
            e1.record()
            barrier_sync()
            if it > 0:
                prefill_ms.append(e0.elapsed_time(e1))
            assert not llm.has_unfinished()
    prefill_ms_max = max(comm.max_scalar(m, dev) if comm else m for m in prefill_ms) if prefill_ms else None
    prefill_ledger = None
    if args.diag and not args.no_prefill_metric:
        from r9700_stack_b200.utils.trace import step_ledger

        llm.add_request(prompt(), SamplingParams(max_tokens=1))
        barrier_sync()
        prefill_ledger = step_ledger(llm, steps=1)
        barrier_sync()

    # ---------------- decode @16 streams ----------------
    total_new = args.warmup + 2 * args.steps + 16
    seqs = [llm.add_request(prompt(), SamplingParams(max_tokens=total_new)) for _ in range(S)]
    while any(not s.prefill_done or not s.output for s in seqs):
        llm.step()
    for _ in range(args.warmup):
        llm.step()
    # count this library's kernel launches in one decode step (eager run of the same step shape)
    lc = _native.launch_counter
    barrier_sync()

    clocks = ClockSampler(_smi_id(dev)) if rank == 0 else None
    if clocks:
        clocks.start()
    # device-timed: CUDA events around each step's graph replay
    llm.runner.device_events = []
    barrier_sync()
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks:
        clocks.mark_start()
    w0.record()
    for _ in range(args.steps):
        llm.step()
    w1.record()
    barrier_sync()
    if clocks:
        clocks.mark_end()
    dev_ms = sum(a.elapsed_time(b) for a, b in llm.runner.device_events)
    e2e_ms = w0.elapsed_time(w1)
    llm.runner.device_events = None
    h2d, d2h = llm.runner.h2d_bytes, llm.runner.d2h_bytes
    clk = clocks.stop() if clocks else None
    dev_ms = comm.max_scalar(dev_ms, dev) if comm else dev_ms
    e2e_ms = comm.max_scalar(e2e_ms, dev) if comm else e2e_ms
    decode16 = S * args.steps / (dev_ms / 1e3)
    e2e16 = S * args.steps / (e2e_ms / 1e3)

    # launch count: an eager run of the decode step shape with the counter on
    from r9700_stack_b200.engine.runner import pack_step
    from r9700_stack_b200.engine.scheduler import ScheduledChunk, SchedulerOutput

    out = SchedulerOutput("decode", [ScheduledChunk(s, s.length - 1, 1, True) for s in seqs])
    lay, arr = pack_step(out, ec.kv_block)
    llm.runner._upload(arr)
    meta = llm.runner.meta.views(lay)
    lc.count, lc.counting = 0, True
    llm.model.forward(meta, llm.runner.ws, lay.T, lay.R)
    lc.counting = False
    launches_per_step = lc.count
    torch.cuda.synchronize(dev)

    diag = None
    if args.diag:
        from r9700_stack_b200.utils.trace import step_ledger

        led = step_ledger(llm, steps=5)
        if comm is not None and world > 1:
            import torch.distributed as dist

            allv = [None] * world
            dist.all_gather_object(allv, led)
            diag = allv
        else:
            diag = [led]

    # ---------------- decode @1 stream: keep one sequence ----------------
    keep = seqs[0]
    for s in seqs[1:]:
        llm.scheduler.running.remove(s)
        llm.scheduler._release(s)
    for _ in range(3):
        llm.step()
    llm.runner.device_events = []
    barrier_sync()
    for _ in range(args.steps):
        llm.step()
    barrier_sync()
    one_ms = sum(a.elapsed_time(b) for a, b in llm.runner.device_events)
    llm.runner.device_events = None
    one_ms = comm.max_scalar(one_ms, dev) if comm else one_ms
    decode1 = args.steps / (one_ms / 1e3)

    if rank == 0:
        res = {
            "metric": METRIC,
            "value": round(decode16, 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": round(decode16 / base16, 3),
            "dtype": ("nvfp4->mxfp4 weights x mxfp8 activations (fp32 accumulate), fp8 KV; reference: mxfp4 x fp8"
                      if args.model == "dense27b" else
                      "experts nvfp4->mxfp4 x mxfp8, attention/GDN/router/shared expert bf16 (fp32 accumulate), fp8 KV"),
            "data": "synthetic: random-init N(0,0.02) weights of the named architecture, uniform random prompt ids",
            "config": {
                "model": ("hybrid-dense-27b (BASELINE config 2: 64 layers 3:1 GDN:GQA, hidden 5120, ffn 17408, vocab 248320)"
                          if args.model == "dense27b" else
                          "hybrid-moe-flashnext (BASELINE config 3: 48 layers 3:1 GDN:GQA, hidden 2048, 288 experts "
                          "top-10 (I=512) + shared expert, vocab 248320; experts NVFP4, rest bf16)"),
                "global_batch": S,
                "seq_len": P,
                "parallelism": f"tp{world}",
                "collectives": "fused GEMM->NVLink push + all-reduce-RMSNorm (decode), NCCL (prefill)" if world > 1 else "none",
                "l2": "inputs larger than L2: every step streams all weights (~15 GB / tp) and the KV cache",
                "layers": cfg.layers,
            },
            "decode_16_streams_tok_s": round(decode16, 2),
            "decode_1_stream_tok_s": round(decode1, 2),
            "prefill_8k_tok_s": round(P / (prefill_ms_max / 1e3), 1) if prefill_ms_max else None,
            "prefill_8k_ms": round(prefill_ms_max, 2) if prefill_ms_max else None,
            "e2e": {"value": round(e2e16, 2), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(launches_per_step * args.steps),
            "gpu_launches_per_step": int(launches_per_step),
            "clocks": clk,
            "build_s": round(build_s, 1),
            "weights_gb_per_rank": round(llm.model.weight_bytes() / 1e9, 2),
        }
        print(json.dumps(res), flush=True)
        if diag is not None:
            print(json.dumps({"diag": {"decode16_ledger_per_rank": diag, "prefill8k_ledger_rank0": prefill_ledger}}),
                  flush=True)
    if comm is not None:
        import torch.distributed as dist

        llm.runner.graphs.clear()
        torch.cuda.synchronize(dev)
        comm.barrier()
        comm.close()
        if dist.is_initialized():
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
