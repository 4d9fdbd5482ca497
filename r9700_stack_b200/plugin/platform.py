"""Platform detection for vLLM's ``vllm.platform_plugins`` group.

``detect()`` returns the qualified name of the B200 platform class when a compute-capability 10.x
device is visible (and ``R9K_PLATFORM`` is not ``0``), else None so vLLM keeps its own choice. The
class extends vLLM's CUDA platform with this framework's device communicator.
Reference: r9700_vllm/platform.py:15-40.
"""
from __future__ import annotations

import os


def _is_b200() -> bool:
    try:
        import torch

        if not torch.cuda.is_available():
            return False
        major, _ = torch.cuda.get_device_capability(0)
        return major == 10
    except Exception:
        return False


def detect() -> str | None:
    if os.environ.get("R9K_PLATFORM", "1") == "0":
        return None
    return "r9700_stack_b200.plugin.platform.B200Platform" if _is_b200() else None


def __getattr__(name):
    # the platform class is built on first use: importing vLLM's CUDA platform needs a driver
    if name == "B200Platform":
        from vllm.platforms.cuda import CudaPlatform

        class B200Platform(CudaPlatform):
            device_name: str = "cuda"

            @classmethod
            def get_device_communicator_cls(cls) -> str:
                return "r9700_stack_b200.plugin.communicator.R9kCommunicator"

        globals()["B200Platform"] = B200Platform
        return B200Platform
    raise AttributeError(name)
