"""``R9K_*`` environment knobs.

Every kernel path has a switch that selects an alternative implementation without a rebuild, in the
spirit of the reference's ``R9K_*=stock`` contract (README.md:144-145): e.g. ``R9K_ATTN=simple``
selects the CUDA-core paged attention instead of the tcgen05 flash-attention kernel, and
``R9K_COMM=nccl`` routes every collective through NCCL. ``R9K_DISABLE=a,b`` lists coarse opt-outs.
Values are read once per process (``refresh()`` re-reads them, for tests).
"""
from __future__ import annotations

import os

_DEFAULTS = {
    "R9K_ATTN": "tc",  # tc | simple
    "R9K_WEIGHT_TILED": "1",  # 1: MX weights stored as contiguous 128x128 units; 0: row-major
    "R9K_GEMM_SK": "0",  # 1: skinny GEMMs use the persistent stream-K kernel
    "R9K_FP4_UNPACK": "0",  # 1: skinny fp4 GEMMs load packed bytes and expand them on chip
    "R9K_GDN_FUSED": "1",  # 1: decode steps run the one-kernel GDN layer core
    "R9K_COMM": "fused",  # fused | nccl
    "R9K_AR_MODE": "pull",  # pull: consumer reads peers' partials; push: GEMM epilogue stores into peers
    "R9K_GDN_STATE": "",  # "" (model default) | bf16 | fp32
    "R9K_DISABLE": "",
    "R9K_AR_ONESHOT_MAX_KB": "512",
    "R9K_AR_QUANT_BITS": "0",  # 4 | 6: lossy WHT-64 compressed all-reduce for large (prefill) messages; 0: exact
    "R9K_AR_QUANT_MIN_KB": "1024",  # smallest message sent compressed
    "R9K_SPIN_TIMEOUT_MS": "1000",
    "R9K_AR_HIST": "0",  # 1: histogram of all-reduce message sizes (utils.trace.AR_HIST)
    "R9K_TRACE": "0",
    "R9K_GEMM_L2PF": "0",  # skinny GEMMs: weight chunks prefetched into L2 beyond the smem ring (0: off; 4-16 measured slower)
    "R9K_MOE_MT": "1",  # 1: grouped skinny MoE GEMMs run several row tiles per CTA (gate/up 2, down 4); 0: one
    "R9K_HC_FUSED": "1",  # 1: one kernel per hyper-connection norm point; 0: logits GEMM + combine_norm + gate_mix  # 1: the runner attaches a utils.trace.DeviceTrace to the model
}
_cache: dict[str, str] = {}


def get(name: str) -> str:
    if name not in _cache:
        _cache[name] = os.environ.get(name, _DEFAULTS.get(name, ""))
    return _cache[name]


def get_int(name: str) -> int:
    return int(get(name) or 0)


def disabled(feature: str) -> bool:
    return feature in {x.strip() for x in get("R9K_DISABLE").split(",") if x.strip()}


def refresh() -> None:
    _cache.clear()


def all_knobs() -> dict[str, str]:
    keys = set(_DEFAULTS) | {k for k in os.environ if k.startswith("R9K_")}
    return {k: get(k) for k in sorted(keys)}
