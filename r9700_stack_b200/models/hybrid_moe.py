"""Hybrid GDN/attention decoder with routed-expert FFNs (Flash-Next class).

FFN block per layer: router GEMM (bf16, fp32 logits) -> moe_route (softmax top-k, renormalised) ->
moe_align (expert-sorted rows, 128-row aligned segments, BN-row work tiles) -> moe_gather (MXFP8 token
rows into sorted order) -> grouped gate/up GEMM with the SwiGLU -> MXFP8 epilogue -> grouped down
GEMM -> moe_combine (router-weighted sum + sigmoid-gated shared expert, one rounding).
Experts are NVFP4 checkpoints converted to MXFP4 at load; attention, router and shared expert bf16.

Expert parallelism: rank r of ``tp_size`` owns experts [r E / tp, (r + 1) E / tp); activations are
replicated, every rank computes its local experts' contributions (plus its TP shard of the shared
expert) and the sublayer's all-reduce sums the partials -- the reference's EP scheme
(r9700_vllm/quant/exl3_moe.py:1-30, r9700_vllm/moe/exl3_combine.py:79-205).
Reference: r9700_vllm/moe/experts.py:84-251, r9700_vllm/moe/shared.py:37-113, r9700_vllm/moe/route.py.
"""
from __future__ import annotations

import torch

from .. import _native
from ..ops import linear as L
from .hybrid import HybridLM, Workspace
from .weights import TPFactory, WeightFactory, from_float


def _ops():
    return _native.ops()


class MoEBuffers:
    """Device buffers of one routed-expert FFN call for up to ``max_tokens`` tokens."""

    def __init__(self, dev, max_tokens: int, hidden: int, n_experts: int, k: int, E_local: int, moe_ffn: int,
                 shared_local: int):
        A = max_tokens * k
        self.moe_act = L.alloc_act(max_tokens, hidden, dev)
        self.logits_e = torch.zeros(max_tokens, n_experts, dtype=torch.float32, device=dev)
        self.ids = torch.zeros(max_tokens, k, dtype=torch.int32, device=dev)
        self.wts = torch.zeros(max_tokens, k, dtype=torch.float32, device=dev)
        self.perm_row = torch.zeros(A, dtype=torch.int32, device=dev)
        self.seg_start = torch.zeros(E_local, dtype=torch.int32, device=dev)
        # sorted rows: 128-row aligned segments, and with token tiles under 128 one 128-row slot per tile
        self.max_rows = A + 256 * min(E_local, A)
        self.max_work = A + E_local
        self.work = torch.zeros(self.max_work, 3, dtype=torch.int32, device=dev)
        self.work_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.sorted_act = L.alloc_act(self.max_rows, hidden, dev)
        self.h_act = L.alloc_act(self.max_rows, moe_ffn, dev)
        self.y_sorted = torch.zeros(self.max_rows, hidden, dtype=torch.bfloat16, device=dev)
        if shared_local:
            self.sh_h = torch.zeros(max_tokens, shared_local, dtype=torch.bfloat16, device=dev)
            self.sh_out = torch.zeros(max_tokens, hidden, dtype=torch.bfloat16, device=dev)
            self.sh_gate = torch.zeros(max_tokens, 1, dtype=torch.float32, device=dev)


def moe_ffn(lay, x: torch.Tensor, mb: MoEBuffers, out: torch.Tensor, *, k: int, e0: int, E_local: int, moe_ffn: int,
            hidden: int, shared_local: int, route_mode: int = 0, bias=None, n_group: int = 1, topk_group: int = 1,
            scale: float = 1.0, renorm: bool = True, remap=None, route: bool = True, gemm_E: int = 0,
            combine: bool = True):
    """Routed experts + shared expert for the T rows of x (bf16) into out (bf16), with the router
    weights applied and summed in one rounding (moe_combine). Experts outside [e0, e0 + E_local)
    belong to other ranks: their rows are skipped and the caller's all-reduce sums the partials.
    ``combine=False`` stops before the combine (the expert rows stay in mb.y_sorted at mb.perm_row)
    and returns the shared expert's output and gate for the caller's own combine."""
    T = x.shape[0]
    o = _ops()
    dev = x.device
    if route:  # (passes over groups of experts reuse the first pass's routing)
        L.bf16_linear(x, lay["router"], out=mb.logits_e[:T], out_dtype=torch.float32)
        o.moe_route(mb.logits_e[:T], k, route_mode, bias, n_group, topk_group, float(scale), renorm, mb.ids[:T],
                    mb.wts[:T])
    A = T * k
    # token tile from the expected rows per active expert (not from T): at T = 64, top-10 over 288
    # experts an expert sees ~2 rows, and 128-token tiles would be almost empty
    per_expert = A / max(1, min(E_local, A))
    BN = 16 if per_expert <= 16 else 32 if per_expert <= 32 else 64 if per_expert <= 64 else 128
    ids = mb.ids[:T] if remap is None else remap(mb.ids[:T])  # expert ids, or cache slot ids
    o.moe_align(ids, e0, E_local, BN, mb.perm_row[:A], mb.seg_start, mb.work, mb.work_count)
    L.quant_act(x, out=mb.moe_act.narrow(T))
    o.moe_gather(mb.moe_act.q[:T], mb.moe_act.sf, k, mb.perm_row[:A], mb.sorted_act.q, mb.sorted_act.sf)
    nwork = min(mb.max_work, -(-A // BN) + min(E_local, A))
    GE = gemm_E or E_local  # experts held by the weight arrays (the work list indexes the first E_local)
    o.gemm_mx_grouped(lay["e_gate"].q, lay["e_gate"].sf, lay["e_up"].q, lay["e_up"].sf, True, mb.sorted_act.q,
                      mb.sorted_act.sf, mb.work[:nwork], mb.work_count, moe_ffn, GE, BN, mb.h_act.q, mb.h_act.sf,
                      _status(dev))
    o.gemm_mx_grouped(lay["e_down"].q, lay["e_down"].sf, None, None, True, mb.h_act.q, mb.h_act.sf, mb.work[:nwork],
                      mb.work_count, hidden, GE, BN, mb.y_sorted, None, _status(dev))
    shared = gate = None
    if shared_local:
        L.bf16_swiglu(x, lay["s_gate"], lay["s_up"], out=mb.sh_h[:T])
        L.bf16_linear(mb.sh_h[:T], lay["s_down"], out=mb.sh_out[:T])
        shared = mb.sh_out[:T]
        if "s_gvec" in lay:
            L.bf16_linear(x, lay["s_gvec"], out=mb.sh_gate[:T], out_dtype=torch.float32)
            gate = mb.sh_gate[:T]
    if not combine:
        return shared, gate
    o.moe_combine(mb.y_sorted, mb.perm_row[:A], mb.wts[:T], k, shared, gate, out)


class MoEWorkspace(Workspace):
    def __init__(self, model: "HybridMoELM", max_tokens: int, max_logit_rows: int):
        super().__init__(model, max_tokens, max_logit_rows)
        c = model.cfg
        self.moe = MoEBuffers(model.device, max_tokens, c.hidden, c.moe_experts, c.moe_topk, model.e_local, c.moe_ffn,
                              model.shared_local)
        if model.placement is not None:
            self.ep_ids = torch.zeros(max_tokens * c.moe_topk, dtype=torch.int32, device=model.device)


class HybridMoELM(HybridLM):
    def __init__(self, cfg, par=None, device="cuda", seed: int = 0, comm=None, placement=None):
        """``placement``: optional expert placement (``parallel.ep_placement``), one list of global
        expert ids per rank; rank r holds placement[r] in that order. Without it rank r holds the
        contiguous range [r E / R, (r + 1) E / R). With a placement every expert's weights are drawn
        from a generator keyed by (layer, expert id), so the model is the same function under any
        placement."""
        tp = (par.tp_size if par is not None else 1)
        assert cfg.moe_experts % tp == 0
        self.placement = None
        if placement is not None:
            from ..parallel.ep_placement import validate

            validate(placement, cfg.moe_experts)
            assert len(placement) == tp, "one expert list per tensor-parallel rank"
            self.placement = [list(map(int, b)) for b in placement]
        self.e_local = cfg.moe_experts // tp
        self.shared_local = cfg.moe_shared_ffn // tp if cfg.moe_shared_ffn else 0
        self.caches = None  # per-layer ExpertCache when experts live in host memory
        super().__init__(cfg, par, device, seed=seed, comm=comm)

    def _build(self, seed: int):
        c = self.cfg
        super()._build(seed)
        r, tp = self.par.tp_rank, self.par.tp_size
        tpf = TPFactory(self.device, seed=seed * 1000 + 77, std=c.init_std)
        wrep = WeightFactory(self.device, seed=seed * 1000 + 79, std=c.init_std)
        H, I = c.hidden, c.moe_ffn
        E, El = c.moe_experts, self.e_local
        mine = self.placement[r] if self.placement is not None else list(range(r * El, (r + 1) * El))
        sl = self.shared_local

        def experts(rows_per, K):
            # every expert of the layer drawn as one stacked [E * rows, K] tensor (one NVFP4 global scale
            # per tensor, as a checkpoint stores it), then this rank's experts in placement order; every
            # expert spans whole 128-row tiles, so tiling the selection gives stack_experts()' unit order
            full = tpf.full(E * rows_per, K)
            sel = full.view(E, rows_per, K)[torch.tensor(mine, device=self.device)].reshape(El * rows_per, K)
            return from_float(sel, "nvfp4", tiled=True, global_from=full)

        for li, lay in enumerate(self.layers):
            lay["router"] = L.BF16Weight(wrep.randn(c.moe_experts, H, dtype=torch.bfloat16))
            lay["e_gate"] = experts(I, H)
            lay["e_up"] = experts(I, H)
            lay["e_down"] = experts(H, I)
            if sl:
                S = c.moe_shared_ffn
                lay["s_gate"] = L.BF16Weight(tpf.raw_rows([(S, r * sl, sl)], H, dtype=torch.bfloat16))
                lay["s_up"] = L.BF16Weight(tpf.raw_rows([(S, r * sl, sl)], H, dtype=torch.bfloat16))
                lay["s_down"] = L.BF16Weight(tpf.full(H, S)[:, r * sl:(r + 1) * sl].to(torch.bfloat16).contiguous())
                lay["s_gvec"] = L.BF16Weight(wrep.randn(1, H, dtype=torch.bfloat16))
            if c.ple_dim:
                lay["ple_gate"] = L.BF16Weight(wrep.randn(c.ple_dim, H, dtype=torch.bfloat16))
                lay["ple_out"] = L.BF16Weight(wrep.randn(H, c.ple_dim, dtype=torch.bfloat16))
        if self.placement is not None:
            # global expert id -> local index on this rank (E_local for experts held elsewhere)
            loc = torch.full((c.moe_experts,), self.e_local, dtype=torch.int32)
            for j, e in enumerate(self.placement[r]):
                loc[e] = j
            self.expert_local = loc.to(self.device)
        self.ple = None
        if c.ple_dim:
            from ..ops.hostmem import HostTable

            # per-layer token embeddings, int6 rows in pinned host memory: row (token * layers + layer)
            self.ple = HostTable.random(c.vocab * c.layers, c.ple_dim, "int6", seed=seed * 7 + 3, std=0.05)

    def local_index(self, e: int) -> int:
        """Local index of global expert e on this rank, or -1 when another rank holds it."""
        if self.placement is None:
            j = e - self.par.tp_rank * self.e_local
            return j if 0 <= j < self.e_local else -1
        row = self.placement[self.par.tp_rank]
        return row.index(e) if e in row else -1

    def _remap_ids(self, ws, T: int):
        k = self.cfg.moe_topk

        def remap(ids):
            out = ws.ep_ids[: T * k]
            torch.index_select(self.expert_local, 0, ids.reshape(-1), out=out)
            return out.view(T, k)

        return remap

    def alloc_workspace(self, max_tokens: int, max_logit_rows: int) -> Workspace:
        ws = MoEWorkspace(self, max_tokens, max_logit_rows)
        if self.caches:
            ws.slot_ids = torch.zeros(max_tokens, self.cfg.moe_topk, dtype=torch.int32, device=self.device)
        if self.ple is not None:
            c = self.cfg
            ws.ple_rows = torch.zeros(max_tokens, c.layers, c.ple_dim, dtype=torch.bfloat16, device=self.device)
            ws.ple_ids = torch.zeros(max_tokens, c.layers, dtype=torch.int64, device=self.device)
            ws.ple_h = torch.zeros(max_tokens, c.ple_dim, dtype=torch.bfloat16, device=self.device)
            ws.ple_lid = torch.arange(c.layers, dtype=torch.int64, device=self.device)
        return ws

    def _embed(self, meta, ws, T: int) -> None:
        super()._embed(meta, ws, T)
        if self.ple is not None:
            # one host gather per step brings every layer's vector of every token
            L_ = self.cfg.layers
            torch.add(meta.input_ids[:T].long().unsqueeze(1) * L_, ws.ple_lid, out=ws.ple_ids[:T])
            self.ple.gather(ws.ple_ids[:T].view(-1), ws.ple_rows[:T].view(-1, self.cfg.ple_dim))

    def _ple(self, i: int, lay, ws, T: int, out: torch.Tensor) -> None:
        """out += (gelu(h W_g^T) * p_i) W_o^T / world -- the per-layer embedding term, added to this
        rank's partial so the sublayer's all-reduce carries it (1/world on every rank)."""
        x = ws.norm_out[:T]
        L.bf16_linear(x, lay["ple_gate"], out=ws.ple_h[:T])
        h = torch.nn.functional.gelu(ws.ple_h[:T], approximate="tanh").mul_(ws.ple_rows[:T, i])
        ws.ple_h[:T].copy_(h)
        L.bf16_linear(ws.ple_h[:T], lay["ple_out"], out=out, residual=out, alpha=1.0 / self.par.tp_size)

    def enable_expert_cache(self, slots: int, profile: str | None = None) -> None:
        """Move every layer's experts to pinned host memory behind a device LRU of `slots` experts.
        ``profile``: a routing profile (safetensors, ``RoutingProfile.save``) whose most routed experts
        of each layer are preloaded (warm start)."""
        from ..ops.expert_cache import ExpertCache, RoutingProfile

        assert self.placement is None, "the expert cache holds contiguous expert ranges"
        prof = RoutingProfile.load(profile) if profile else None
        e0 = self.par.tp_rank * self.e_local
        self.caches = []
        for i, lay in enumerate(self.layers):
            cache = ExpertCache(lay["e_gate"], lay["e_up"], lay["e_down"], self.e_local, slots, self.device)
            del lay["e_gate"], lay["e_up"], lay["e_down"]
            if prof is not None:
                cache.warm_ids = prof.top(i, slots, e0, self.e_local)
                cache.warm(cache.warm_ids)
            self.caches.append(cache)
        torch.cuda.empty_cache()

    def record_routing(self, enable: bool = True) -> None:
        """Start (or stop) recording every layer's routed experts into ``self.routing_profile``."""
        from ..ops.expert_cache import RoutingProfile

        if enable:
            self.routing_profile = RoutingProfile(len(self.layers), self.cfg.moe_experts, self.device)
        else:
            self.routing_profile = None

    def _ffn_block(self, i, lay, meta, ws: MoEWorkspace, T: int, call: int, fused: bool) -> None:
        c = self.cfg
        out = self._reduce_target(ws, T, call, fused)
        mode = 0 if c.moe_router == "softmax" else 1
        if self.caches is None and self.placement is not None:
            moe_ffn(lay, ws.norm_out[:T], ws.moe, out, k=c.moe_topk, e0=0, E_local=self.e_local, moe_ffn=c.moe_ffn,
                    hidden=c.hidden, shared_local=self.shared_local, route_mode=mode, remap=self._remap_ids(ws, T))
        elif self.caches is None:
            moe_ffn(lay, ws.norm_out[:T], ws.moe, out, k=c.moe_topk, e0=self.par.tp_rank * self.e_local,
                    E_local=self.e_local, moe_ffn=c.moe_ffn, hidden=c.hidden, shared_local=self.shared_local,
                    route_mode=mode)
        else:
            cache = self.caches[i]
            g, u, d = cache.weights
            lay_c = dict(lay, e_gate=g, e_up=u, e_down=d)
            e0 = self.par.tp_rank * self.e_local
            if T * c.moe_topk <= cache.S:
                # every expert this step can route to fits: device LRU + copies of the misses
                moe_ffn(lay_c, ws.norm_out[:T], ws.moe, out, k=c.moe_topk, e0=0, E_local=cache.S, moe_ffn=c.moe_ffn,
                        hidden=c.hidden, shared_local=self.shared_local, route_mode=mode,
                        remap=lambda ids: (cache.route(ids, e0, ws.slot_ids[:T]), ws.slot_ids[:T])[1])
            else:
                # wider batches (prefill): stream the experts through the slots in groups of S; each
                # pass parks its expert rows in token-pair order, one combine sums them all (the same
                # order and single rounding as resident experts)
                A = T * c.moe_topk
                pair = getattr(ws, "moe_pair", None)
                if pair is None or pair.shape[0] < A + 1:
                    ws.moe_pair = pair = torch.zeros(A + 1, c.hidden, dtype=torch.bfloat16, device=self.device)
                    ws.moe_ident = torch.arange(A, dtype=torch.int32, device=self.device)
                ident = ws.moe_ident[:A]
                mb = ws.moe
                shared = gate = None
                for p, grp in enumerate(cache.stream_groups()):
                    n = cache.warm(grp)
                    sg = moe_ffn(lay_c, ws.norm_out[:T], mb, out, k=c.moe_topk, e0=0, E_local=n,
                                 moe_ffn=c.moe_ffn, hidden=c.hidden, shared_local=self.shared_local if p == 0 else 0,
                                 route_mode=mode, route=p == 0, gemm_E=cache.S, combine=False,
                                 remap=lambda ids: cache.slots_for(ids, e0, ws.slot_ids[:T]))
                    if p == 0:
                        shared, gate = sg
                    src = mb.perm_row[:A].long()
                    dest = torch.where(src >= 0, ident.long(), torch.full_like(src, A))  # row A: discard
                    pair.index_copy_(0, dest, mb.y_sorted[src.clamp(min=0)])
                _ops().moe_combine(pair, ident, mb.wts[:T], c.moe_topk, shared, gate, out)
        if getattr(self, "routing_profile", None) is not None:
            self.routing_profile.record(i, ws.moe.ids[:T])
        if self.ple is not None:
            self._ple(i, lay, ws, T, out)
        self._after_partial(ws, T, call, fused)


def _status(dev):
    from ..utils import status

    return status.status(dev)
