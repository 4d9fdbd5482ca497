"""Fake (meta) implementations of the ``torch.ops.r9k`` ops for tracing.

Every compute op of the library writes into caller-provided outputs and returns nothing, so its fake
implementation has nothing to compute: shapes and aliasing are carried by the schema's ``(a!)``
annotations. Host-side helper ops (symmetric-memory setup) are not traceable and are skipped.
"""
from __future__ import annotations

import torch

HOST_OPS = {"symm_alloc", "symm_free", "symm_ipc_handle", "symm_open", "symm_close", "symm_view",
            "symm_collective_region_bytes", "p2p_probe", "gemm_trace", "gdn_chunk_trace"}
_done: set[str] = set()


def op_names() -> list[str]:
    """Names of the library's ops, from the loaded schemas."""
    from .. import _native

    _native.load_library()
    names = set()
    for s in torch._C._jit_get_all_schemas():
        if s.name.startswith("r9k::"):
            names.add(s.name.split("::", 1)[1])
    return sorted(names)


def register_fakes() -> int:
    n = 0
    for name in op_names():
        if name in HOST_OPS or name in _done:
            continue
        qual = f"r9k::{name}"
        try:
            torch.library.register_fake(qual)(lambda *args, **kwargs: None)
        except RuntimeError:
            pass  # already has a fake / meta kernel
        _done.add(name)
        n += 1
    return n
