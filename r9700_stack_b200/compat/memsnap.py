"""Memory audit: per-category device memory of a built engine and the caching allocator's state.

``engine_memory(llm)`` splits resident bytes into weights, KV cache, recurrent state, workspace and
speculative buffers; ``allocator_summary()`` condenses ``torch.cuda.memory_stats``; ``snapshot(path)``
dumps the allocator's segment snapshot for offline inspection. Reference: r9700_vllm/compat/memsnap.py
(per-module activation peak + allocator snapshot).
"""
from __future__ import annotations

import pickle

import torch


def _tensor_bytes(obj, seen) -> int:
    n = 0
    if isinstance(obj, torch.Tensor):
        if obj.is_cuda and obj.data_ptr() not in seen:
            seen.add(obj.data_ptr())
            n += obj.numel() * obj.element_size()
    elif isinstance(obj, dict):
        for v in obj.values():
            n += _tensor_bytes(v, seen)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            n += _tensor_bytes(v, seen)
    elif hasattr(obj, "__dict__") and not isinstance(obj, type):
        for v in vars(obj).values():
            n += _tensor_bytes(v, seen)
    return n


def engine_memory(llm) -> dict:
    seen: set[int] = set()
    m = llm.model
    out = {
        "weights": _tensor_bytes({"embed": getattr(m, "embed", None), "layers": getattr(m, "layers", None),
                                  "lm_head": getattr(m, "lm_head", None)}, seen),
        "kv_cache": _tensor_bytes([getattr(m, "kv", None), getattr(m, "lat", None), getattr(m, "icache", None)], seen),
        "recurrent_state": _tensor_bytes([getattr(m, "ssm", None), getattr(m, "conv", None)], seen),
        "workspace": _tensor_bytes(llm.runner.ws, seen),
    }
    out["total_gb"] = round(sum(out.values()) / 1e9, 3)
    return out


def allocator_summary(device=None) -> dict:
    s = torch.cuda.memory_stats(device)
    keys = ["allocated_bytes.all.current", "allocated_bytes.all.peak", "reserved_bytes.all.current",
            "num_alloc_retries", "num_ooms"]
    return {k: s.get(k, 0) for k in keys}


def snapshot(path: str) -> None:
    with open(path, "wb") as f:
        pickle.dump(torch.cuda.memory_snapshot(), f)
