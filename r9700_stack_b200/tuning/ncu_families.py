"""Summarise an ncu launch list (``--metrics gpu__time_duration.sum --csv``) by kernel family.

    python -m r9700_stack_b200.tuning.ncu_families launches.csv [--steps N]

Prints a markdown table: family, launches, total device time, share, and per-step figures when the
capture covered N identical steps. The families follow the reference's profile binning
(profiling/analyze-prof.py: expert_moe, attention, gdn, allreduce_comm, ...).
"""
from __future__ import annotations

import argparse
import csv
import re
from collections import defaultdict

FAMILIES = [
    ("gemm_tcgen05", r"gemm_tc_kernel|gemm_sk_kernel"),
    ("attention", r"attn|attention"),
    ("gdn", r"gdn_"),
    ("moe_glue", r"moe_"),
    ("norm/quant", r"rmsnorm|quant|norm_rope|qk_norm"),
    ("allreduce_comm", r"ar_|allreduce|push|nccl|Nccl"),
    ("spec", r"spec_"),
    ("torch", r"at::|void at_|elementwise|index|reduce_kernel|gather|scatter|copy|fill"),
]


def family(name: str) -> str:
    for fam, pat in FAMILIES:
        if re.search(pat, name):
            return fam
    return "other"


def summarise(path: str, steps: int = 1) -> str:
    tot = defaultdict(float)
    cnt = defaultdict(int)
    by_kernel = defaultdict(float)
    with open(path) as f:
        lines = [l for l in f if l.startswith('"')]
    rows = list(csv.reader(lines))
    hdr = rows[0]
    ik, im, iv = hdr.index("Kernel Name"), hdr.index("Metric Name"), hdr.index("Metric Value")
    unit_i = hdr.index("Metric Unit") if "Metric Unit" in hdr else None
    for r in rows[1:]:
        if r[im] != "gpu__time_duration.sum":
            continue
        v = float(r[iv].replace(",", ""))
        unit = r[unit_i] if unit_i is not None else "ns"
        us = v / 1000.0 if unit in ("ns", "nsecond") else (v * 1000.0 if unit in ("ms", "msecond") else v)
        fam = family(r[ik])
        tot[fam] += us
        cnt[fam] += 1
        by_kernel[r[ik].split("(")[0][:70]] += us
    all_us = sum(tot.values())
    out = ["| family | launches/step | us/step | share |", "|---|---|---|---|"]
    for fam in sorted(tot, key=lambda x: -tot[x]):
        out.append(f"| {fam} | {cnt[fam] / steps:.0f} | {tot[fam] / steps:.1f} | {100 * tot[fam] / all_us:.1f}% |")
    out.append(f"| **total** | {sum(cnt.values()) / steps:.0f} | {all_us / steps:.1f} | 100% |")
    out += ["", "| kernel (top 12) | us/step |", "|---|---|"]
    for k in sorted(by_kernel, key=lambda x: -by_kernel[x])[:12]:
        out.append(f"| `{k}` | {by_kernel[k] / steps:.1f} |")
    return "\n".join(out)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("csv")
    ap.add_argument("--steps", type=int, default=1)
    a = ap.parse_args(argv)
    print(summarise(a.csv, a.steps))


if __name__ == "__main__":
    main()

