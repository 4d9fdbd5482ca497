"""Version gate: warns when the runtime differs from the versions this build was tested with.

The kernels target sm_100a with CUDA 12.9 and PyTorch 2.11; the serving front end and the vLLM
plugin were exercised with vLLM 0.22. ``check()`` returns a list of warnings (empty when every
component matches) and logs them once. Reference: r9700_vllm/compat/gate.py:14-46 (tested vLLM pins
per monkeypatch).
"""
from __future__ import annotations

import logging

log = logging.getLogger("r9700_stack_b200")

TESTED = {"torch": "2.11", "cuda": "12.9", "vllm": "0.22", "compute_capability": (10, 0)}
_warned = False


def _ver(mod: str) -> str | None:
    try:
        m = __import__(mod)
        return getattr(m, "__version__", None)
    except Exception:
        return None


def check(log_once: bool = True) -> list[str]:
    global _warned
    import torch

    w = []
    tv = torch.__version__
    if not tv.startswith(TESTED["torch"]):
        w.append(f"torch {tv} (tested {TESTED['torch']})")
    cv = torch.version.cuda or "none"
    if torch.cuda.is_available() and not cv.startswith("12"):
        w.append(f"CUDA runtime {cv} (tested {TESTED['cuda']})")
    vv = _ver("vllm")
    if vv is not None and not vv.startswith(TESTED["vllm"]):
        w.append(f"vllm {vv} (tested {TESTED['vllm']})")
    if torch.cuda.is_available():
        cc = torch.cuda.get_device_capability(0)
        if cc != TESTED["compute_capability"]:
            w.append(f"compute capability {cc} (kernels are built for sm_100a)")
    if w and log_once and not _warned:
        for m in w:
            log.warning("r9700_stack_b200 untested: %s", m)
        _warned = True
    return w
