"""Host model of the pull protocol the NVLink collectives run (for CPU-rank tests).

Each rank owns a region in shared host memory: per buffer a flag word and a data slot. Call g uses
buffer g % 2 and epoch g + 1: a rank writes its contribution into its own slot, publishes the epoch
in its own flag, waits (bounded) until every peer's flag reaches the epoch, then reads the peers'
slots and reduces them in rank order. A rank that stops publishing makes the others' waits run out,
which surfaces as :class:`ProtocolTimeout` -- the host-side analogue of the kernels' status word.
This is the same state machine as ``csrc/collectives.cu`` and the fused decode all-reduce, so the
epoch / double-buffer reasoning can be exercised with real process scheduling skew on CPU ranks.
(reference: the CPU-rank protocol tests called for by its race test, tests/test_ar_race.py:1-16.)
"""
from __future__ import annotations

import time

import torch


class ProtocolTimeout(RuntimeError):
    pass


class SimRegions:
    """flags [world, 2] int64 and data [world, 2, n] float64 in shared memory."""

    def __init__(self, world: int, n: int):
        self.flags = torch.zeros(world, 2, dtype=torch.int64).share_memory_()
        self.data = torch.zeros(world, 2, n, dtype=torch.float64).share_memory_()


class SimRank:
    def __init__(self, regions: SimRegions, rank: int, world: int, timeout_s: float = 2.0):
        self.r, self.rank, self.world, self.timeout_s = regions, rank, world, timeout_s
        self.seq = 0

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        g = self.seq
        b, epoch = g & 1, g + 1
        self.r.data[self.rank, b].copy_(x)
        self.r.flags[self.rank, b] = epoch  # publish after the data (the release store)
        t0 = time.monotonic()
        for p in range(self.world):
            while int(self.r.flags[p, b]) < epoch:
                if time.monotonic() - t0 > self.timeout_s:
                    raise ProtocolTimeout(f"rank {self.rank}: peer {p} did not publish call {g}")
                time.sleep(0)
        out = torch.zeros_like(self.r.data[0, b])
        for p in range(self.world):  # rank order: bit-identical on every rank
            out += self.r.data[p, b]
        self.seq += 1
        return out
