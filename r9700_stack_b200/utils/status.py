"""Device status words.

Kernels that wait (on an mbarrier, a peer flag or a sequence counter) bound every wait with a
``%globaltimer`` deadline. When a wait gives up the kernel writes ``{code, kernel id, block, detail}``
into a per-device int32[4] status buffer and returns, so the CUDA context stays usable. The host reads
the buffer at safe points (between steps) with :func:`check` and raises :class:`DeviceWaitError`.
Reference counterpart: the spin-timeout diagnostic record of kernels/r9k_ar.hip:1133-1180, which the
reference follows with a trap; here the kernel returns instead.
"""
from __future__ import annotations

import torch

_STATUS: dict[int, torch.Tensor] = {}

ERR_NAMES = {0: "ok", 1: "mbarrier timeout", 2: "peer timeout", 3: "bounds", 4: "config"}


class DeviceWaitError(RuntimeError):
    pass


def status(device: torch.device | int | None = None) -> torch.Tensor:
    if device is None:
        device = torch.cuda.current_device()
    if isinstance(device, str):
        device = torch.device(device)
    if isinstance(device, torch.device):
        idx = device.index if device.index is not None else torch.cuda.current_device()
    else:
        idx = int(device)
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=f"cuda:{idx}")
        _STATUS[idx] = t
    return t


def check(device=None, reset: bool = True) -> None:
    s = status(device)
    vals = s.tolist()
    if vals[0] != 0:
        if reset:
            s.zero_()
        raise DeviceWaitError(
            f"device wait failed: {ERR_NAMES.get(vals[0], vals[0])} kernel={vals[1]} block={vals[2]} detail={vals[3]}"
        )
