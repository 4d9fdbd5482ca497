"""Tensor-parallel communicators.

* :class:`NcclComm` - ``torch.distributed`` over NCCL (NVLink / NVSwitch, NVLS when NCCL picks it).
  This is the baseline and the fallback for every collective the fused kernels decline; it plays the
  role RCCL plays under the reference's custom collectives (r9700_vllm/comm/r4d_ar.py:178-188).
* The fused NVLink kernels (symmetric memory, one-shot / two-shot / GEMM-fused) live in
  :mod:`r9700_stack_b200.parallel.symm` and plug in through the same two methods.

All methods are CUDA-graph capturable (no host sync, no allocation after warm-up).
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def init_distributed(timeout_s: int = 120) -> tuple[int, int, int]:
    """Initialise the default process group from torchrun's environment (one process per GPU)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        kw = dict(backend=backend, timeout=timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local


class NcclComm:
    def __init__(self, group=None):
        self.group = group
        if dist.is_initialized():
            self.world_size = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:  # single process: collectives are identities
            self.world_size, self.rank = 1, 0
        self._gather_bufs: dict[tuple, torch.Tensor] = {}

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world_size > 1:
            from ..utils.trace import note_all_reduce

            note_all_reduce(t.numel() * t.element_size())
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather_lastdim(self, t: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[R, n] per rank -> [R, world * n] (rank-major along the last dim)."""
        if self.world_size == 1:
            if out is not None:
                out.copy_(t)
                return out
            return t
        R, n = t.shape
        key = (R, n, t.dtype)
        buf = self._gather_bufs.get(key)
        if buf is None:
            buf = torch.empty(self.world_size, R, n, dtype=t.dtype, device=t.device)
            self._gather_bufs[key] = buf
        dist.all_gather_into_tensor(buf, t.contiguous(), group=self.group)
        res = buf.permute(1, 0, 2).reshape(R, self.world_size * n)
        if out is not None:
            out.copy_(res)
            return out
        return res

    def barrier(self) -> None:
        if self.world_size > 1:
            dist.barrier(group=self.group)

    def max_scalar(self, x: float, device) -> float:
        if self.world_size == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())
