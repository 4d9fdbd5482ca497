"""MoE experts resident in pinned host memory behind a per-layer device LRU cache.

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

    def stats(self) -> dict:
        h, m = (int(x) for x in self.counters.tolist())
        return {"hits": h, "misses": m, "hit_rate": h / max(1, h + m), "slots": self.S, "experts": self.E}
