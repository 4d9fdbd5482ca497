"""``R9K_*`` environment knobs.

Every kernel path has a switch that selects an alternative implementation without a rebuild, in the
spirit of the reference's ``R9K_*=stock`` contract (README.md:144-145): every knob accepts the value
``stock``, which selects the simplest path this library has for that step (a CUDA-core kernel instead
of the tcgen05 one, the unfused kernel sequence instead of the fused one, NCCL instead of the NVLink
kernels). There is no vLLM stock path under this engine, so "stock" means the baseline path here.
``R9K_DISABLE=a,b`` lists coarse opt-outs. Values are read once per process (``refresh()`` re-reads
them, for tests).
"""
from __future__ import annotations

import os

# name -> (default, value that "stock" selects, meaning)
_KNOBS = {
    "R9K_ATTN": ("tc", "simple", "tc: tcgen05 flash attention; simple: CUDA-core paged attention"),
    "R9K_ATTN_DEC": ("1", "0", "1: keys-on-M split-KV decode attention; 0: the row-tile kernel"),
    "R9K_INDEXER": ("tc", "simple", "tc: lightning-indexer / QSA group scores on tcgen05 (keys on M, heads on N); "
                    "simple: the CUDA-core kernel"),
    "R9K_MLA_ATTN": ("tc", "simple", "tc: sparse MLA attention on tcgen05 (selected keys on the MMA's M side, heads on "
                     "N; the pipelined gather/MMA/softmax kernel when the grid fills two CTAs per SM, else the "
                     "single-stage one); tc1: always the single-stage kernel; simple: the CUDA-core kernel"),
    "R9K_WEIGHT_TILED": ("1", "0", "1: MX weights stored as contiguous 128x128 units; 0: row-major"),
    "R9K_GEMM_SK": ("0", "0", "1: skinny GEMMs use the persistent stream-K kernel"),
    "R9K_GEMM_SWAP": ("1", "0", "1: prefill-sized MX GEMMs put tokens on the MMA's M side (vector epilogue); 0: weight rows"),
    "R9K_GEMM_CLUSTER": ("1", "0", "1: split-K GEMM tiles reduce over distributed shared memory (cluster); 0: global fix-up"),
    "R9K_FP4_UNPACK": ("0", "0", "1: skinny fp4 GEMMs load packed bytes and expand them on chip"),
    "R9K_GDN_FUSED": ("1", "0", "1: decode steps run the one-kernel GDN layer core"),
    "R9K_GDN_PREFILL": ("chunked", "serial",
                        "chunked: prefill runs the tcgen05 chunked delta rule (WY form, 128-token chunks); serial: "
                        "the token-serial recurrence"),
    "R9K_GDN_CHUNK_MIN": ("256", "256", "fewest tokens in a step's longest sequence that take the chunked GDN prefill"),
    "R9K_GDN_PREFETCH": ("0", "0", "1: decode steps prefetch each GDN layer's recurrent state into L2 during its in_proj GEMM "
                         "(measured slower: 16-stream decode 2207 vs 2250 tok/s)"),
    "R9K_COMM": ("fused", "nccl", "fused: NVLink kernels fused into GEMMs / norms; nccl: every collective on NCCL"),
    "R9K_AR_MODE": ("ll", "pull", "ll: GEMM epilogue stores epoch-tagged partials into peers, consumer polls its own "
                    "memory; pull: consumer reads peers' partials; push: plain stores + per-tile flags"),
    "R9K_GDN_STATE": ("", "", "'' (model default) | bf16 | fp32"),
    "R9K_DISABLE": ("", "", "comma list of coarse opt-outs (e.g. plugin)"),
    "R9K_AR_ONESHOT_MAX_KB": ("512", "512", "largest standalone all-reduce sent one-shot"),
    "R9K_AR_QUANT_BITS": ("0", "0", "4 | 6: lossy WHT-64 compressed all-reduce for large (prefill) messages; 0: exact"),
    "R9K_AR_QUANT_MIN_KB": ("1024", "1024", "smallest message sent compressed"),
    "R9K_PREFILL_AR": ("symm", "nccl", "symm: prefill all-reduces on the NVLink two-shot kernel; nccl: NCCL"),
    "R9K_LOGITS_AG": ("symm", "nccl", "symm: logits all-gather on the NVLink kernel; nccl: NCCL"),
    "R9K_SPIN_TIMEOUT_MS": ("1000", "1000", "bound of every device-side wait"),
    "R9K_AR_HIST": ("0", "0", "1: histogram of all-reduce message sizes (utils.trace.AR_HIST)"),
    "R9K_TRACE": ("0", "0", "1: the runner attaches a utils.trace.DeviceTrace to the model"),
    "R9K_GEMM_L2PF": ("0", "0", "skinny GEMMs: weight chunks prefetched into L2 beyond the smem ring (0: off)"),
    "R9K_MOE_MT": ("1", "0", "1: grouped skinny MoE GEMMs run several row tiles per CTA; 0: one"),
    "R9K_HC_FUSED": ("1", "0", "1: one kernel per hyper-connection norm point; 0: logits GEMM + combine_norm + gate_mix"),
    "R9K_NVFP4": ("mxfp4", "mxfp4", "mxfp4: NVFP4 checkpoints convert to MXFP4 at load; native: served as NVFP4"),
    "R9K_EP": ("ar", "ar", "ar: experts' partials summed by the all-reduce; a2a: all-to-all dispatch/combine"),
}
# knobs the C++ library reads with getenv (kept in sync by export_native)
_NATIVE = ("R9K_ATTN_DEC", "R9K_INDEXER", "R9K_MLA_ATTN", "R9K_FP4_UNPACK", "R9K_GEMM_L2PF", "R9K_GEMM_SK", "R9K_MOE_MT", "R9K_GEMM_CLUSTER",
           "R9K_GEMM_SWAP")
_DEFAULTS = {k: v[0] for k, v in _KNOBS.items()}
_cache: dict[str, str] = {}


def get(name: str) -> str:
    if name not in _cache:
        v = os.environ.get(name, _DEFAULTS.get(name, ""))
        if v.strip().lower() == "stock" and name in _KNOBS:
            v = _KNOBS[name][1]
        _cache[name] = v
    return _cache[name]


def get_int(name: str) -> int:
    return int(get(name) or 0)


def disabled(feature: str) -> bool:
    return feature in {x.strip() for x in get("R9K_DISABLE").split(",") if x.strip()}


def refresh() -> None:
    _cache.clear()


def export_native() -> None:
    """Resolve ``stock`` for the knobs the kernel library reads itself (before it loads)."""
    for k in _NATIVE:
        if os.environ.get(k, "").strip().lower() == "stock":
            os.environ[k] = _KNOBS[k][1]


def describe() -> dict[str, str]:
    return {k: v[2] for k, v in _KNOBS.items()}


def all_knobs() -> dict[str, str]:
    keys = set(_DEFAULTS) | {k for k in os.environ if k.startswith("R9K_")}
    return {k: get(k) for k in sorted(keys)}
