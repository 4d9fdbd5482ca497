"""MoE experts resident in pinned host memory behind a per-layer device LRU cache.

Warm start: ``warm(experts)`` preloads a layer's most wanted experts, taken from a routing profile
(``RoutingProfile``: per-layer expert counts recorded while serving, saved as safetensors next to the
model), so the first steps after start-up do not pay the misses of an empty cache (reference:
r9700_vllm/moe/cache.py:79,246, model-expertprofile.safetensors).

``ExpertCache`` takes a layer's stacked expert weights (gate, up, down as tiled MX matrices), moves
them to page-locked host memory and keeps ``slots`` experts on the device in the same layout, so the
grouped GEMM runs on the slot arrays with slot ids in place of expert ids. Each step ``route()``
runs the device LRU (``lru_route``) and the host -> device copies of the misses (``expert_copy``,
through the UVA mapping) -- two launches, no host synchronisation, capturable in a CUDA graph.
Hit / miss counters stay on the device; ``stats()`` reads them.
Reference: r9700_vllm/moe/cache.py:182-414 (LayerCache: host backing store + VRAM arena of S slots,
update / stage_cold, stats), kernels/third_party/davetha/r4d_lru.hip.
"""
from __future__ import annotations

import torch

from .. import _native
from . import linear as L


def _per_expert(w: L.MXWeight, E: int) -> tuple[int, int]:
    return w.q.numel() // E, w.sf.numel() // E


class ExpertCache:
    def __init__(self, gate: L.MXWeight, up: L.MXWeight, down: L.MXWeight, E: int, slots: int, device):
        assert 1 <= slots <= min(E, 1024)
        self.E, self.S, self.device = E, slots, torch.device(device)
        self.host, self.dev, self.bytes, self.views = [], [], [], []
        for w in (gate, up, down):
            qb, sb = _per_expert(w, E)
            assert qb % 16 == 0 and sb % 16 == 0
            hq = torch.empty(w.q.numel(), dtype=torch.uint8, pin_memory=True)
            hq.copy_(w.q.reshape(-1).cpu())
            hs = torch.empty(w.sf.numel(), dtype=torch.uint8, pin_memory=True)
            hs.copy_(w.sf.reshape(-1).cpu())
            dq = torch.zeros(slots * qb, dtype=torch.uint8, device=self.device)
            ds = torch.zeros(slots * sb, dtype=torch.uint8, device=self.device)
            self.host += [hq, hs]
            self.dev += [dq, ds]
            self.bytes += [qb, sb]
            rows_e = w.N // E
            self.views.append(L.MXWeight(dq.view(-1, *w.q.shape[1:]), ds, w.fp4, rows_e * slots, w.K))
        dev = self.device
        self.slot_of = torch.full((E,), -1, dtype=torch.int32, device=dev)
        self.expert_of = torch.full((slots,), -1, dtype=torch.int32, device=dev)
        self.stamp = torch.zeros(slots, dtype=torch.int64, device=dev)
        self.clock = torch.zeros(1, dtype=torch.int64, device=dev)
        self.miss_e = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.miss_s = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.miss_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counters = torch.zeros(2, dtype=torch.int64, device=dev)  # hits, misses
        self.warm_ids: list[int] = []  # the warm-start set: streamed last, so it stays resident

    @property
    def weights(self) -> tuple[L.MXWeight, L.MXWeight, L.MXWeight]:
        return tuple(self.views)

    @property
    def host_bytes(self) -> int:
        return sum(t.numel() for t in self.host)

    @property
    def device_bytes(self) -> int:
        return sum(t.numel() for t in self.dev)

    def route(self, ids: torch.Tensor, e0: int, slot_ids: torch.Tensor) -> None:
        """ids: routed expert ids [T, k] (global); writes slot ids [T, k] (S + 1 = not local)."""
        from ..utils import status

        ops = _native.ops()
        ops.lru_route(ids, e0, self.E, self.S, self.slot_of, self.expert_of, self.stamp, self.clock, self.miss_e,
                      self.miss_s, self.miss_count, self.counters, slot_ids, status.status(self.device))
        ops.expert_copy(self.host, self.dev, self.bytes, self.miss_e, self.miss_s, self.miss_count, self.S)

    def load_range(self, g0: int) -> int:
        """Copy experts [g0, g0 + S) (clipped) into slots 0.. with one copy per region, and make the
        LRU maps describe that content. Returns the number of experts loaded."""
        n = min(self.S, self.E - g0)
        for h, d, b in zip(self.host, self.dev, self.bytes):
            d[: n * b].copy_(h[g0 * b:(g0 + n) * b], non_blocking=True)
        self.slot_of.fill_(-1)
        self.slot_of[g0:g0 + n] = torch.arange(n, dtype=torch.int32, device=self.device)
        self.expert_of.fill_(-1)
        self.expert_of[:n] = torch.arange(g0, g0 + n, dtype=torch.int32, device=self.device)
        self.stamp.fill_(0)
        return n

    def warm(self, experts) -> int:
        """Warm start: copy the given experts (local ids, most wanted first; e.g. the top of a routing
        profile) into slots 0.. and make the LRU maps describe that content, older stamps for later
        entries so the least wanted leave first. Returns the number loaded."""
        ids = [int(e) for e in experts][: self.S]
        n = len(ids)
        self.slot_of.fill_(-1)
        self.expert_of.fill_(-1)
        if n:
            # one gather launch over UVA (the miss-copy kernel with the whole list as misses)
            t = torch.tensor(ids, dtype=torch.int64).to(self.device, non_blocking=True)
            self.miss_e[:n].copy_(t)
            self.miss_s[:n].copy_(torch.arange(n, dtype=torch.int32, device=self.device))
            self.miss_count.fill_(n)
            _native.ops().expert_copy(self.host, self.dev, self.bytes, self.miss_e, self.miss_s, self.miss_count, self.S)
            self.miss_count.fill_(0)
            self.slot_of[t] = torch.arange(n, dtype=torch.int32, device=self.device)
            self.expert_of[:n] = t.int()
            self.stamp[:n] = torch.arange(n, 0, -1, dtype=torch.int64, device=self.device)
        self.stamp[n:] = 0
        self.clock.fill_(n + 1)
        return n

    def stream_groups(self) -> list[list[int]]:
        """Expert groups (local ids, at most S each) for a wide batch that streams every expert through
        the slots: the warm-start set, when there is one, goes last so it is what stays resident."""
        warm = set(self.warm_ids)
        rest = [e for e in range(self.E) if e not in warm]
        groups = [rest[i:i + self.S] for i in range(0, len(rest), self.S)]
        return groups + ([list(self.warm_ids)] if self.warm_ids else [])

    def slots_for(self, ids: torch.Tensor, e0: int, out: torch.Tensor) -> torch.Tensor:
        """Slot of each routed expert id [T, k] (global ids; -1 where the expert is not in a slot)."""
        local = ids.long() - e0
        ok = (local >= 0) & (local < self.E)
        s = self.slot_of[local.clamp(0, self.E - 1)]
        out.copy_(torch.where(ok, s, torch.full_like(s, -1)))
        return out

    def stats(self) -> dict:
        h, m = (int(x) for x in self.counters.tolist())
        return {"hits": h, "misses": m, "hit_rate": h / max(1, h + m), "slots": self.S, "experts": self.E}


class RoutingProfile:
    """Per-layer expert routing counts: recorded on the device while enabled (one index_add per MoE
    layer per step, no host synchronisation), saved to / loaded from a safetensors file
    ``{"layer.{i}": int64 [E]}``."""

    def __init__(self, layers: int, E: int, device):
        self.counts = torch.zeros(layers, E, dtype=torch.int64, device=device)

    def record(self, layer: int, ids: torch.Tensor) -> None:
        flat = ids.reshape(-1).long()
        self.counts[layer].index_add_(0, flat, torch.ones_like(flat))

    def top(self, layer: int, n: int, e0: int = 0, E_local: int | None = None) -> list[int]:
        """The n most routed experts of a layer among [e0, e0 + E_local), as local ids, most first."""
        c = self.counts[layer].cpu()
        E_local = E_local or c.numel()
        loc = c[e0:e0 + E_local]
        order = torch.argsort(loc, descending=True, stable=True)
        return [int(i) for i in order[:n]]

    def save(self, path: str) -> None:
        from safetensors.torch import save_file

        save_file({f"layer.{i}": self.counts[i].cpu().contiguous() for i in range(self.counts.shape[0])}, path)

    @classmethod
    def load(cls, path: str, device="cpu") -> "RoutingProfile":
        from safetensors.torch import load_file

        d = load_file(path)
        layers = sorted(int(k.split(".")[1]) for k in d)
        p = cls(len(layers), d[f"layer.{layers[0]}"].numel(), device)
        for i in layers:
            p.counts[i].copy_(d[f"layer.{i}"])
        return p
