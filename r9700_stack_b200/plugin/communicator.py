"""vLLM device communicator whose all-reduce uses this framework's NVLink collectives.

Tensor-parallel all-reduces of bf16 tensors that fit the symmetric slot go through
``SymmCollectives`` (one-shot or two-shot, picked by the start-up calibration); everything else, and
any size the calibration found NCCL faster for, goes to vLLM's CUDA communicator (NCCL). Collective
set-up is all-or-nothing: if any rank fails to build its region, every rank keeps NCCL.
Reference: r9700_vllm/comm/r4d_ar.py:130-188 (R9kCommunicator), comm/r9k_ar.py:422-439.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _base():
    from vllm.distributed.device_communicators.cuda_communicator import CudaCommunicator

    return CudaCommunicator


class R9kCommunicator(_base()):  # type: ignore[misc]
    def __init__(self, cpu_group, device=None, device_group=None, unique_name: str = ""):
        super().__init__(cpu_group, device, device_group, unique_name)
        self.r9k = None
        ok = 1
        try:
            if self.world_size > 1:
                from ..parallel.collectives import SymmCollectives

                self.r9k = SymmCollectives(self.device, group=self.device_group)
                self.r9k.calibrate()
        except Exception:
            ok = 0
        flag = torch.tensor([ok], dtype=torch.int32)
        if self.world_size > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=cpu_group)
        if int(flag) == 0:
            self.r9k = None

    def all_reduce(self, input_):
        c = self.r9k
        if c is not None and c.fits(input_) and c.should("all_reduce", input_.numel() * 2) != "nccl":
            out = input_.clone()
            return c.all_reduce(out)
        return super().all_reduce(input_)
