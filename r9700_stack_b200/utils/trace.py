"""Tracing: device-side time stamps inside the model's forward, a step ledger from the torch profiler,
and the all-reduce message-size histogram.

* ``DeviceTrace`` writes ``%globaltimer`` into a device buffer at named points of the forward (one
  1-thread kernel per mark, in stream order). The marks are captured into decode CUDA graphs like any
  kernel, so replayed steps are traced too, with no profiler attached: durations are the time between
  consecutive marks, attributed to the later one (e.g. ``L3.attn`` = layer 3's norm + attention + its
  all-reduce). Enable with ``model.trace = DeviceTrace(device)`` or ``R9K_TRACE=1`` (the runner
  attaches one). Reference: the device stage stamps of r9k_ar8_fused_t / R9K_MHC_PROF.
* ``step_ledger(llm, steps)`` runs engine steps under the torch profiler (CUPTI) and bins every
  kernel by family (``tuning.ncu_families.family``): per-step device milliseconds per family, the
  sum of kernel time and the host wall time of the steps. Reference: bench/ds41/ledger/ledger.py.
  As the reference measured, a profiler stretches the step: read kernel durations, not periods.
* ``AR_HIST``: message sizes of every all-reduce (power-of-two bins) when ``R9K_AR_HIST=1``
  (reference: R9K_AR_HIST in comm/r9k_ar.py).
"""
from __future__ import annotations

import re
import time
from collections import Counter, defaultdict

import torch

from .. import knobs

AR_HIST: Counter = Counter()


def note_all_reduce(nbytes: int) -> None:
    if knobs.get("R9K_AR_HIST") == "1":
        AR_HIST[1 << max(0, (int(nbytes) - 1).bit_length())] += 1


class DeviceTrace:
    def __init__(self, device, max_marks: int = 8192):
        self.device = torch.device(device)
        self.buf = torch.zeros(max_marks, dtype=torch.int64, device=self.device)
        self.names: list[str] = []
        self._n = 0

    def begin(self) -> None:
        self._n = 0
        self.names = []

    def mark(self, name: str) -> None:
        if self._n >= self.buf.numel():
            return
        from .. import _native

        _native.ops().trace_stamp(self.buf, self._n)
        self.names.append(name)
        self._n += 1

    def read(self) -> list[tuple[str, float]]:
        """(mark, microseconds since the previous mark) of the last traced forward or replay."""
        torch.cuda.synchronize(self.device)
        t = self.buf[: len(self.names)].cpu().tolist()
        return [(self.names[i], (t[i] - t[i - 1]) / 1e3) for i in range(1, len(t))]

    def summary(self) -> dict:
        """Microseconds per category (the mark name without its layer prefix) and the total."""
        cat = defaultdict(float)
        rows = self.read()
        for name, us in rows:
            cat[re.sub(r"^L\d+\.", "", name)] += us
        return {"total_us": round(sum(us for _, us in rows), 1)} | {k: round(v, 1) for k, v in sorted(cat.items())}


def step_ledger(llm, steps: int = 5) -> dict:
    """Profile `steps` engine steps; device ms per step by kernel family."""
    from torch.profiler import ProfilerActivity, profile

    from ..tuning.ncu_families import family

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            if not llm.has_unfinished():
                break
            llm.step()
        torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    fam = defaultdict(float)
    kernels = defaultdict(float)
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            us = ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
            fam[family(ev.name)] += us
            kernels[ev.name] += us
    n = max(1, steps)
    top = sorted(kernels.items(), key=lambda kv: -kv[1])[:10]
    return {
        "steps": steps,
        "wall_ms_per_step": round(wall * 1e3 / n, 3),
        "kernel_ms_per_step": round(sum(fam.values()) / 1e3 / n, 3),
        "by_family_ms_per_step": {k: round(v / 1e3 / n, 3) for k, v in sorted(fam.items(), key=lambda kv: -kv[1])},
        "top_kernels_ms_per_step": {k[:80]: round(v / 1e3 / n, 3) for k, v in top},
    }
