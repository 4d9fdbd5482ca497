"""NVLink SHARP (NVLS) collectives: all-reduce and all-gather through an NVSwitch multicast object.

The buffer is torch's symmetric memory (``torch.distributed._symmetric_memory``: one allocation per
rank mapped into every peer and bound to a multicast object when the switch supports it); the
kernels are this library's (``csrc/nvls.cu``): ``multimem.ld_reduce`` sums a slice across all GPUs
inside the switch, ``multimem.st`` writes the result to every GPU at once. ``available`` is False
where the platform has no multicast (the caller keeps NCCL).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _native
from ..utils import status as _status


class NvlsComm:
    def __init__(self, device, group=None, capacity_bytes: int = 96 << 20, timeout_s: float = 2.0):
        import torch.distributed._symmetric_memory as symm_mem

        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.timeout_s = timeout_s
        self.capacity = capacity_bytes
        self.buf = symm_mem.empty(capacity_bytes, dtype=torch.uint8, device=self.device)
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        self.mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        self.local = int(self.buf.data_ptr())
        self.sig = torch.tensor([int(p) for p in self.handle.signal_pad_ptrs], dtype=torch.int64)
        self.sig_slots = int(symm_mem.get_signal_pad_size()) // 4
        # one [sequence, ticket] pair for every collective of this object: they share the signal pads,
        # so their barrier epochs must come from one increasing sequence
        self.seq = torch.zeros(2, dtype=torch.int32, device=self.device)
        # every rank must agree (a rank without multicast makes the whole group fall back)
        ok = torch.tensor([1 if self.mc else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        self.available = bool(int(ok))

    def fits_all_reduce(self, t: torch.Tensor) -> bool:
        n = t.numel()
        return (self.available and t.dtype == torch.bfloat16 and t.is_contiguous() and n % (8 * self.world) == 0
                and n * 2 <= self.capacity and t.data_ptr() % 16 == 0)

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        _native.ops().nvls_all_reduce(t, t, self.mc, self.local, self.capacity, self.sig, self.sig_slots, self.rank,
                                      self.world, self.seq, _status.status(self.device), self.timeout_s)
        return t

    def fits_all_gather(self, t: torch.Tensor) -> bool:
        b = t.numel() * t.element_size()
        return (self.available and t.element_size() == 4 and t.is_contiguous() and b % 16 == 0
                and b * self.world <= self.capacity and t.data_ptr() % 16 == 0)

    def all_gather(self, t: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out [W, *t.shape] (rank-major)."""
        _native.ops().nvls_all_gather(t, out, self.mc, self.local, self.capacity, self.sig, self.sig_slots,
                                      self.rank, self.world, self.seq, _status.status(self.device), self.timeout_s)
        return out
