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
from .weights import WeightFactory, from_float


def _ops():
    return _native.ops()


class MoEWorkspace(Workspace):
    def __init__(self, model: "HybridMoELM", max_tokens: int, max_logit_rows: int):
        super().__init__(model, max_tokens, max_logit_rows)
        c, dev = model.cfg, model.device
        k, El = c.moe_topk, model.e_local
        A = max_tokens * k
        self.moe_act = L.alloc_act(max_tokens, c.hidden, dev)
        self.logits_e = torch.zeros(max_tokens, c.moe_experts, dtype=torch.float32, device=dev)
        self.ids = torch.zeros(max_tokens, k, dtype=torch.int32, device=dev)
        self.wts = torch.zeros(max_tokens, k, dtype=torch.float32, device=dev)
        self.perm_row = torch.zeros(A, dtype=torch.int32, device=dev)
        self.seg_start = torch.zeros(El, dtype=torch.int32, device=dev)
        self.max_rows = A + 128 * min(El, A)
        self.max_work = A + El
        self.work = torch.zeros(self.max_work, 3, dtype=torch.int32, device=dev)
        self.work_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.sorted_act = L.alloc_act(self.max_rows, c.hidden, dev)
        self.h_act = L.alloc_act(self.max_rows, c.moe_ffn, dev)
        self.y_sorted = torch.zeros(self.max_rows, c.hidden, dtype=torch.bfloat16, device=dev)
        if model.shared_local:
            self.sh_h = torch.zeros(max_tokens, model.shared_local, dtype=torch.bfloat16, device=dev)
            self.sh_out = torch.zeros(max_tokens, c.hidden, dtype=torch.bfloat16, device=dev)
            self.sh_gate = torch.zeros(max_tokens, 1, dtype=torch.float32, device=dev)


class HybridMoELM(HybridLM):
    def __init__(self, cfg, par=None, device="cuda", seed: int = 0, comm=None):
        tp = (par.tp_size if par is not None else 1)
        assert cfg.moe_experts % tp == 0
        self.e_local = cfg.moe_experts // tp
        self.shared_local = cfg.moe_shared_ffn // tp if cfg.moe_shared_ffn else 0
        super().__init__(cfg, par, device, seed=seed, comm=comm)

    def _build(self, seed: int):
        c = self.cfg
        super()._build(seed)
        r = self.par.tp_rank
        wf = WeightFactory(self.device, seed=seed * 1000 + 77 + r, std=c.init_std)
        wrep = WeightFactory(self.device, seed=seed * 1000 + 79, std=c.init_std)
        H, I = c.hidden, c.moe_ffn
        for lay in self.layers:
            lay["router"] = L.BF16Weight(wrep.randn(c.moe_experts, H, dtype=torch.bfloat16))
            # the local experts of a layer are generated and quantised as one stacked [E * rows, K] tensor
            # (one NVFP4 global scale per layer); tiling the stacked tensor gives exactly the unit order
            # of stack_experts() over per-expert weights, since every expert spans whole 128-row tiles
            El = self.e_local
            lay["e_gate"] = from_float(wf.randn(El * I, H), "nvfp4", tiled=True)
            lay["e_up"] = from_float(wf.randn(El * I, H), "nvfp4", tiled=True)
            lay["e_down"] = from_float(wf.randn(El * H, I), "nvfp4", tiled=True)
            if self.shared_local:
                lay["s_gate"] = L.BF16Weight(wf.randn(self.shared_local, H, dtype=torch.bfloat16))
                lay["s_up"] = L.BF16Weight(wf.randn(self.shared_local, H, dtype=torch.bfloat16))
                lay["s_down"] = L.BF16Weight(wf.randn(H, self.shared_local, dtype=torch.bfloat16))
                lay["s_gvec"] = L.BF16Weight(wrep.randn(1, H, dtype=torch.bfloat16))

    def alloc_workspace(self, max_tokens: int, max_logit_rows: int) -> Workspace:
        return MoEWorkspace(self, max_tokens, max_logit_rows)

    def _ffn_block(self, i, lay, meta, ws: MoEWorkspace, T: int, call: int, fused: bool) -> None:
        c = self.cfg
        k = c.moe_topk
        o = _ops()
        x = ws.norm_out[:T]  # bf16 output of the post-attention norm
        L.bf16_linear(x, lay["router"], out=ws.logits_e[:T], out_dtype=torch.float32)
        o.moe_route(ws.logits_e[:T], k, 0 if c.moe_router == "softmax" else 1, None, 1, 1, 1.0, True,
                    ws.ids[:T], ws.wts[:T])
        BN = 16 if T <= 16 else 128
        A = T * k
        o.moe_align(ws.ids[:T], self.par.tp_rank * self.e_local, self.e_local, BN, ws.perm_row[:A], ws.seg_start,
                    ws.work, ws.work_count)
        L.quant_act(x, out=ws.moe_act.narrow(T))
        o.moe_gather(ws.moe_act.q[:T], ws.moe_act.sf, k, ws.perm_row[:A], ws.sorted_act.q, ws.sorted_act.sf)
        nwork = min(ws.max_work, -(-A // BN) + self.e_local)
        o.gemm_mx_grouped(lay["e_gate"].q, lay["e_gate"].sf, lay["e_up"].q, lay["e_up"].sf, True, ws.sorted_act.q,
                          ws.sorted_act.sf, ws.work[:nwork], ws.work_count, c.moe_ffn, self.e_local, BN,
                          ws.h_act.q, ws.h_act.sf, _status(self.device))
        o.gemm_mx_grouped(lay["e_down"].q, lay["e_down"].sf, None, None, True, ws.h_act.q, ws.h_act.sf,
                          ws.work[:nwork], ws.work_count, c.hidden, self.e_local, BN, ws.y_sorted, None,
                          _status(self.device))
        shared = gate = None
        if self.shared_local:
            L.bf16_swiglu(x, lay["s_gate"], lay["s_up"], out=ws.sh_h[:T])
            L.bf16_linear(ws.sh_h[:T], lay["s_down"], out=ws.sh_out[:T])
            L.bf16_linear(x, lay["s_gvec"], out=ws.sh_gate[:T], out_dtype=torch.float32)
            shared, gate = ws.sh_out[:T], ws.sh_gate[:T]
        out = self._reduce_target(ws, T, call, fused)
        o.moe_combine(ws.y_sorted, ws.perm_row[:A], ws.wts[:T], k, shared, gate, out)
        self._after_partial(ws, T, call, fused)


def _status(dev):
    from ..utils import status

    return status.status(dev)
