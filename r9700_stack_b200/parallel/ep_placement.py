"""Expert placement for expert-parallel MoE: which rank holds which experts.

With experts sharded over the ranks, a decode step is as slow as its busiest rank. At decode sizes an
expert's cost is streaming its weights, paid once per step if any token routes to it, so a rank's
load is the number of DISTINCT local experts its tokens touch; at prefill sizes it is the number of
(token, expert) rows. Routing is skewed (a few experts take most tokens), so contiguous ranges
[r E / R, (r + 1) E / R) can leave one rank with most of the hot experts.

* ``profile(ids, E)``: per-expert routing frequencies from recorded top-k ids (a routing profile).
* ``skew(p, placement, tokens, k)``: the skew model. For routing probabilities p (sum 1 per token
  choice) and a step of ``tokens`` tokens with top-k, expert e is touched with probability
  ``1 - (1 - p_e) ** (tokens * k)``; a rank's expected load is the sum over its experts. Returns
  per-rank loads, the max / mean imbalance and the same for row counts.
* ``place(p, ranks, tokens, k)``: equal-size placement (every rank holds E / R experts, so stacked
  expert weights keep one shape) that minimises the max expected load: longest-processing-time
  greedy on the expected loads, then pairwise swaps between the busiest rank and the others while
  the max load drops.
* ``save`` / ``load``: the placement as JSON (``{"ranks": R, "experts": E, "placement": [[ids]...]}``).

Reference: bench/ds41/epskew/skew_model.py and skew_place.py (CPU skew model and placement search),
moe/exl3_placement.py:18 (placement JSON sidecar).
"""
from __future__ import annotations

import json

import numpy as np


def contiguous(E: int, ranks: int) -> list[list[int]]:
    n = E // ranks
    return [list(range(r * n, (r + 1) * n)) for r in range(ranks)]


def profile(ids, E: int) -> np.ndarray:
    """Routing frequencies [E] (sum 1) from top-k expert ids of any shape (negative ids ignored)."""
    a = np.asarray(ids).reshape(-1)
    a = a[(a >= 0) & (a < E)]
    c = np.bincount(a, minlength=E).astype(np.float64)
    return c / max(c.sum(), 1.0)


def touch_prob(p: np.ndarray, tokens: int, k: int) -> np.ndarray:
    return 1.0 - np.power(1.0 - np.clip(p, 0.0, 1.0), tokens * k)


def skew(p: np.ndarray, placement: list[list[int]], tokens: int, k: int) -> dict:
    p = np.asarray(p, dtype=np.float64)
    t = touch_prob(p, tokens, k)
    load = np.array([t[ex].sum() for ex in placement])
    rows = np.array([p[ex].sum() * tokens * k for ex in placement])
    return {
        "touched_per_rank": load.tolist(),
        "imbalance": float(load.max() / max(load.mean(), 1e-12)),
        "rows_per_rank": rows.tolist(),
        "row_imbalance": float(rows.max() / max(rows.mean(), 1e-12)),
    }


def place(p, ranks: int, tokens: int = 16, k: int = 8) -> list[list[int]]:
    p = np.asarray(p, dtype=np.float64)
    E = p.shape[0]
    assert E % ranks == 0, "experts must divide evenly over the ranks"
    cap = E // ranks
    w = touch_prob(p, tokens, k)
    order = np.argsort(-w, kind="stable")
    bins: list[list[int]] = [[] for _ in range(ranks)]
    load = np.zeros(ranks)
    for e in order:
        open_ = [r for r in range(ranks) if len(bins[r]) < cap]
        r = min(open_, key=lambda i: (load[i], i))
        bins[r].append(int(e))
        load[r] += w[e]
    # pairwise swaps from the busiest rank while they lower the max load
    for _ in range(4 * E):
        hi = int(np.argmax(load))
        best = None
        for lo in range(ranks):
            if lo == hi:
                continue
            for a in bins[hi]:
                for b in bins[lo]:
                    d = w[a] - w[b]
                    if d <= 0:
                        continue
                    new_max = max(load[hi] - d, load[lo] + d)
                    others = max((load[r] for r in range(ranks) if r not in (hi, lo)), default=0.0)
                    m = max(new_max, others)
                    if m < load.max() - 1e-12 and (best is None or m < best[0]):
                        best = (m, lo, a, b, d)
        if best is None:
            break
        _, lo, a, b, d = best
        bins[hi][bins[hi].index(a)] = b
        bins[lo][bins[lo].index(b)] = a
        load[hi] -= d
        load[lo] += d
    return [sorted(b) for b in bins]


def validate(placement: list[list[int]], E: int) -> None:
    flat = sorted(e for b in placement for e in b)
    if flat != list(range(E)):
        raise ValueError("placement must hold every expert exactly once")
    if len({len(b) for b in placement}) != 1:
        raise ValueError("every rank must hold the same number of experts")


def save(path: str, placement: list[list[int]]) -> None:
    E = sum(len(b) for b in placement)
    validate(placement, E)
    with open(path, "w") as f:
        json.dump({"ranks": len(placement), "experts": E, "placement": placement}, f)


def load(path: str) -> list[list[int]]:
    with open(path) as f:
        d = json.load(f)
    validate(d["placement"], d["experts"])
    if len(d["placement"]) != d["ranks"]:
        raise ValueError("placement rank count mismatch")
    return d["placement"]
