"""Build and load the in-tree sm_100a kernel library.

The CUDA/C++ sources under ``csrc/`` compile into one torch extension ``r9k_C`` whose ops live in
``torch.ops.r9k``. The shared object is written inside the package (``_build/``), never into a
user cache, so a copy of the tree carries its kernels with it. A hash of the sources is stored next
to the library; a stale or missing library is rebuilt on load.

On a machine with a CUDA device the library is mandatory: :func:`ops` raises if it cannot be built
or loaded, so no code path silently falls back to PyTorch.
"""
from __future__ import annotations

import glob
import hashlib
import os
import threading

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC_DIR = os.path.join(PKG_DIR, "csrc")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
EXT_NAME = "r9k_C"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-DNDEBUG",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fno-strict-aliasing",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]

_lock = threading.Lock()
_loaded = False


def sources() -> list[str]:
    srcs = sorted(glob.glob(os.path.join(CSRC_DIR, "*.cu")) + glob.glob(os.path.join(CSRC_DIR, "*.cpp")))
    return srcs


def _source_hash() -> str:
    h = hashlib.sha256()
    for p in sorted(glob.glob(os.path.join(CSRC_DIR, "*"))):
        if os.path.isfile(p):
            h.update(os.path.basename(p).encode())
            with open(p, "rb") as f:
                h.update(f.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def lib_path() -> str:
    return os.path.join(BUILD_DIR, EXT_NAME + ".so")


def _stamp_path() -> str:
    return os.path.join(BUILD_DIR, EXT_NAME + ".srchash")


def is_current() -> bool:
    if not os.path.exists(lib_path()) or not os.path.exists(_stamp_path()):
        return False
    with open(_stamp_path()) as f:
        return f.read().strip() == _source_hash()


def build(verbose: bool = False) -> str:
    """Compile every CUDA source for sm_100a into ``_build/r9k_C.so`` (cross-compiles without a GPU)."""
    from torch.utils.cpp_extension import load

    os.makedirs(BUILD_DIR, exist_ok=True)
    # keep torch from adding its own -gencode list: the explicit sm_100a flags above are the only target
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    load(
        name=EXT_NAME,
        sources=sources(),
        extra_cflags=CXX_FLAGS,
        extra_cuda_cflags=NVCC_FLAGS,
        extra_include_paths=[CSRC_DIR],
        build_directory=BUILD_DIR,
        verbose=verbose,
        is_python_module=False,
        with_cuda=True,
    )
    with open(_stamp_path(), "w") as f:
        f.write(_source_hash())
    return lib_path()


def load_library(rebuild_if_stale: bool = True) -> None:
    """Load the kernel library into ``torch.ops.r9k`` (building it first when missing or stale)."""
    global _loaded
    with _lock:
        if _loaded:
            return
        from . import knobs

        knobs.export_native()
        if not is_current():
            if not rebuild_if_stale and os.path.exists(lib_path()):
                pass
            else:
                build()
        torch.ops.load_library(lib_path())
        _loaded = True


def available() -> bool:
    try:
        load_library()
        return True
    except Exception:  # pragma: no cover - reported by ops()
        return False


class _LaunchCounter:
    """Proxy over ``torch.ops.r9k`` that counts op calls while ``counting`` is set.

    Every op of the library launches exactly one kernel, so the count is the number of this
    library's kernel launches (used by the benchmark's ``gpu_launches`` field)."""

    def __init__(self):
        self.counting = False
        self.count = 0

    def __getattr__(self, name):
        fn = getattr(torch.ops.r9k, name)
        if not self.counting:
            return fn

        def wrapped(*a, **k):
            self.count += 1
            return fn(*a, **k)

        return wrapped


launch_counter = _LaunchCounter()


def ops():
    """``torch.ops.r9k`` with the native library loaded; raises if it cannot be."""
    if not _loaded:
        load_library()
    return launch_counter
