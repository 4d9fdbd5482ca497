"""Standalone NVLink collectives on a symmetric region, with NCCL as the fallback and the baseline.

``SymmCollectives`` owns one CUDA-IPC region per rank and runs, in one kernel each, a one-shot
all-reduce, an all-gather and a reduce-scatter (``csrc/collectives.cu``); a two-shot all-reduce is a
reduce-scatter followed by an all-gather. Every call advances a device-resident sequence counter, so
calls replay inside CUDA graphs. ``should(op, nbytes)`` picks the algorithm per message size from a
table measured at start-up by :meth:`calibrate` (graph-timed candidates, the MAX over ranks decides,
as in the reference's calibration: r9700_vllm/comm/calibrate.py:1-35, :120-184); messages larger than
the slot go to NCCL. Reference: r9700_vllm/comm/r9k_ar.py:261-601 (one-shot / two-shot / all-gather).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _native
from ..utils import status as _status

AR, AG, RS = 0, 1, 2
CHUNK = 4096


class SymmCollectives:
    def __init__(self, device, group=None, slot_bytes: int = 16 << 20, timeout_s: float = 2.0):
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.slot_bytes = slot_bytes
        self.timeout_s = timeout_s
        ops = _native.ops()
        nbytes = int(ops.symm_collective_region_bytes(slot_bytes))
        self.local_ptr = int(ops.symm_alloc(nbytes))
        handle = ops.symm_ipc_handle(self.local_ptr).numpy().tobytes()
        handles = [handle]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
        ptrs, self._opened = [], []
        for i, h in enumerate(handles):
            if i == self.rank:
                ptrs.append(self.local_ptr)
            else:
                p = int(ops.symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
                self._opened.append(p)
                ptrs.append(p)
        self.peers = torch.tensor(ptrs, dtype=torch.int64)
        self.seq = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.table: dict[tuple[str, int], str] = {}
        if self.world > 1:
            dist.barrier(group=group)

    # -------------------------------------------------------------------------------------------
    def _run(self, mode: int, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        _native.ops().symm_collective(mode, x, out, self.peers, self.rank, self.world, self.slot_bytes, self.seq,
                                      _status.status(self.device), float(self.timeout_s))
        return out

    def fits(self, x: torch.Tensor) -> bool:
        return x.dtype == torch.bfloat16 and x.numel() * 2 <= self.slot_bytes and x.numel() <= 16384 * CHUNK

    def all_reduce_oneshot(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x = x.contiguous()
        return self._run(AR, x.view(-1), (out if out is not None else torch.empty_like(x)).view(-1)).view(x.shape)

    def reduce_scatter(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x = x.contiguous().view(-1)
        out = out if out is not None else torch.empty(x.numel() // self.world, dtype=x.dtype, device=x.device)
        return self._run(RS, x, out.view(-1))

    def all_gather(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """out = concat over ranks of x (flattened, rank-major)."""
        x = x.contiguous().view(-1)
        out = out if out is not None else torch.empty(x.numel() * self.world, dtype=x.dtype, device=x.device)
        return self._run(AG, x, out.view(-1))

    def all_reduce_twoshot(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x = x.contiguous()
        seg = self.reduce_scatter(x)
        res = out if out is not None else torch.empty_like(x)
        self.all_gather(seg, res.view(-1))
        return res

    def wht_ok(self, x: torch.Tensor, bits: int) -> bool:
        n = x.numel()
        return (x.dtype == torch.bfloat16 and n % 64 == 0 and x.data_ptr() % 16 == 0
                and -(-n // CHUNK) * (64 * 8 * bits + 128) <= (self.slot_bytes // self.world) & ~15)

    def all_reduce_wht(self, x: torch.Tensor, bits: int = 6, out: torch.Tensor | None = None,
                       phase: int = 3) -> torch.Tensor:
        """Lossy compressed all-reduce: WHT-64 rotation, 4- or 6-bit codes with a bf16 scale per 64
        elements, reduced in the rotated domain; bit-identical on every rank (``parallel.compress``
        restates it in torch)."""
        x = x.contiguous()
        out = out if out is not None else torch.empty_like(x)
        _native.ops().symm_ar_wht(x.view(-1), out.view(-1), self.peers, self.rank, self.world, self.slot_bytes,
                                  self.seq, _status.status(self.device), float(self.timeout_s), int(bits), int(phase))
        return out

    def twoshot_ok(self, x: torch.Tensor) -> bool:
        return x.numel() % (self.world * CHUNK) == 0

    # -------------------------------------------------------------------------------------------
    def should(self, op: str, nbytes: int) -> str:
        """'oneshot' | 'twoshot' | 'nccl' for an `op` of nbytes (calibrated table, else a size rule)."""
        if nbytes > self.slot_bytes:
            return "nccl"
        b = 1 << max(12, (nbytes - 1).bit_length())
        if (op, b) in self.table:
            return self.table[(op, b)]
        if op == "all_reduce":
            return "oneshot" if nbytes <= (1 << 20) else "twoshot"
        return "oneshot"

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        """In-place all-reduce of x (bf16) by the calibrated algorithm; with ``R9K_AR_QUANT_BITS`` set
        (4 or 6), messages of at least ``R9K_AR_QUANT_MIN_KB`` go through the lossy compressed path."""
        from .. import knobs

        bits = knobs.get_int("R9K_AR_QUANT_BITS")
        if (self.world > 1 and bits in (4, 6) and x.numel() * 2 >= knobs.get_int("R9K_AR_QUANT_MIN_KB") * 1024
                and self.wht_ok(x, bits)):
            x.copy_(self.all_reduce_wht(x, bits))
            return x
        algo = self.should("all_reduce", x.numel() * x.element_size()) if self.fits(x) else "nccl"
        if algo == "twoshot" and not self.twoshot_ok(x):
            algo = "oneshot"
        if algo == "nccl" or self.world == 1:
            if self.world > 1:
                dist.all_reduce(x, group=self.group)
            return x
        y = self.all_reduce_twoshot(x) if algo == "twoshot" else self.all_reduce_oneshot(x)
        x.copy_(y)
        return x

    def calibrate(self, sizes=(8 << 10, 64 << 10, 512 << 10, 2 << 20, 8 << 20), iters: int = 20) -> dict:
        """Graph-time each candidate per size on every rank; the slowest rank's time decides."""
        res = {}
        for nbytes in sizes:
            if nbytes > self.slot_bytes:
                continue
            n = nbytes // 2
            n -= n % (self.world * CHUNK) if n >= self.world * CHUNK else 0
            x = torch.randn(max(n, 1), device=self.device).bfloat16()
            cands = {"oneshot": lambda: self.all_reduce_oneshot(x)}
            if self.twoshot_ok(x):
                cands["twoshot"] = lambda: self.all_reduce_twoshot(x)
            if self.world > 1:
                cands["nccl"] = lambda: dist.all_reduce(x.clone(), group=self.group)
            times = {}
            for name, fn in cands.items():
                fn()
                torch.cuda.synchronize(self.device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    fn()
                e1.record()
                torch.cuda.synchronize(self.device)
                t = torch.tensor([e0.elapsed_time(e1) / iters], device=self.device)
                if self.world > 1:
                    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
                times[name] = float(t)
            best = min(times, key=times.get)
            self.table[("all_reduce", 1 << max(12, (nbytes - 1).bit_length()))] = best
            res[nbytes] = {k: round(v * 1e3, 2) for k, v in times.items()} | {"best": best}
        return res

    def close(self) -> None:
        ops = _native.ops()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            ops.symm_close(p)
        self._opened = []
        if self.local_ptr:
            ops.symm_free(self.local_ptr)
            self.local_ptr = 0
