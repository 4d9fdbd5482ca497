"""One-layer draft models that run on the target's kernels: the MTP head and the block drafter.

Both are a single decoder layer (gated attention + FFN, or routed MoE when the target is MoE) with the
target's embedding table and lm_head shared by reference, and their own paged KV cache indexed by
the target's block tables. They differ only in what enters the layer:

* MTP (``kind="mtp"``, Qwen3-Next / DeepSeek multi-token prediction, applied k times with shared
  weights): input at position p is ``fc([enorm(embed(x_{p+1})), hnorm(h_p)])`` where h_p is the
  target's final residual at p (or, for the 2nd..k-th draft, the drafter's own output at p).
* Block drafter (``kind="block"``, DFlash-style): context positions carry ``fc([0, hnorm(h_p)])``;
  a proposal block is the last accepted token followed by mask tokens, all attending to the whole
  context and to each other (non-causal within the block), and the mask positions' logits are the
  drafts of one forward pass.

Reference: r9700_vllm/models/dflash.py:26-230 (fp8 DFlash drafter), r9700_vllm/models/qwen4_exp.py:61
(MTP layer, fp8 -> MXFP4 requant), r9700_vllm/spec/mtp_rocm.py:21-57.
"""
from __future__ import annotations

import torch

from ..models.config import HybridConfig, ParallelConfig
from ..models.hybrid import HybridLM, StepMeta, Workspace
from ..models.weights import WeightFactory
from ..ops import linear as L


class _Unfused:
    """A view of a communicator that never takes the fused path."""

    fused = False

    def __init__(self, comm):
        self._c = comm
        self.world_size = getattr(comm, "world_size", 1)
        self.rank = getattr(comm, "rank", 0)

    def all_reduce_(self, t):
        return self._c.all_reduce_(t)

    def all_gather_lastdim(self, t, out=None):
        return self._c.all_gather_lastdim(t, out=out)


def draft_config(target: HybridConfig) -> HybridConfig:
    """The drafter layer's config: one full-attention layer of the target's shapes, fp8 weights."""
    return target.scaled(name=target.name + "-draft", layers=1, full_attn_interval=1, weight_format="mxfp8"
                         if target.weight_format != "bf16" else "bf16", mtp_layers=0, drafter="")


def _draft_base(target_model):
    from ..models.hybrid_moe import HybridMoELM

    return HybridMoELM if isinstance(target_model, HybridMoELM) else HybridLM


def build_draft_model(target_model, kind: str, seed: int = 0):
    """A draft model class derived from the target's class (dense or MoE) with the drafter input stage."""
    base = _draft_base(target_model)

    class DraftLM(base):  # type: ignore[misc, valid-type]
        def __init__(self):
            self.kind = kind
            self.target = target_model
            cfg = draft_config(target_model.cfg)
            # the drafter's row-parallel outputs reduce through the plain (NCCL) path of the target's
            # communicator; the fused per-step protocol belongs to the target's forward
            super().__init__(cfg, target_model.par, target_model.device, seed=seed + 101,
                             comm=_Unfused(target_model.comm))

        def _build(self, s: int):
            super()._build(s)
            c, t = self.cfg, self.target
            # shared with the target (the reference's MTP layers share embed / lm_head too)
            self.embed = t.embed
            self.lm_head = t.lm_head
            wf = WeightFactory(self.device, seed=s * 1000 + 555, std=c.init_std)
            H = c.hidden
            self.enorm = wf.norm(H, c.norm_plus_one)
            self.hnorm = wf.norm(H, c.norm_plus_one)
            self.fc = L.BF16Weight(wf.randn(H, 2 * H, dtype=torch.bfloat16))
            self.mask_embed = wf.randn(1, H, dtype=torch.bfloat16)
            self.h_src = None  # [rows, H] bf16 hidden rows the next forward reads
            self.h_idx = None  # [T] int32 row of h_src per token
            self.row_kind = None  # [T] int32: 0 token row, 1 mask row, -1 context row (block drafter)

        def alloc_workspace(self, max_tokens: int, max_logit_rows: int) -> Workspace:
            ws = super().alloc_workspace(max_tokens, max_logit_rows)
            H = self.cfg.hidden
            ws.cat_in = torch.zeros(max_tokens, 2 * H, dtype=torch.bfloat16, device=self.device)
            ws.h_rows = torch.zeros(max_tokens, H, dtype=torch.bfloat16, device=self.device)
            ws.e_rows = torch.zeros(max_tokens, H, dtype=torch.bfloat16, device=self.device)
            ws.h_out = torch.zeros(max_logit_rows, H, dtype=torch.bfloat16, device=self.device)
            return ws

        def _embed(self, meta: StepMeta, ws: Workspace, T: int) -> None:
            c, H = self.cfg, self.cfg.hidden
            torch.index_select(self.embed, 0, meta.input_ids[:T], out=ws.e_rows[:T])
            torch.index_select(self.h_src, 0, self.h_idx[:T], out=ws.h_rows[:T])
            kind = self.row_kind[:T].unsqueeze(1)
            if self.kind == "block":
                ws.e_rows[:T].copy_(torch.where(kind == 1, self.mask_embed, ws.e_rows[:T]))
            L.rmsnorm(ws.e_rows[:T], self.enorm, c.rms_eps, plus_one=c.norm_plus_one, out=ws.cat_in[:T, :H])
            L.rmsnorm(ws.h_rows[:T], self.hnorm, c.rms_eps, plus_one=c.norm_plus_one, out=ws.cat_in[:T, H:])
            if self.kind == "block":
                # context rows carry only the target's feature, block rows only their token embedding
                ws.cat_in[:T, :H].masked_fill_(kind < 0, 0)
                ws.cat_in[:T, H:].masked_fill_(kind >= 0, 0)
            L.bf16_linear(ws.cat_in[:T], self.fc, out=ws.resid[:T])

        def forward(self, meta: StepMeta, ws: Workspace, T: int, R: int) -> torch.Tensor:
            logits = super().forward(meta, ws, T, R)
            # the drafter's own pre-norm output rows feed the next MTP draft
            torch.index_select(ws.resid[:T], 0, meta.logits_idx[:R], out=ws.h_out[:R])
            return logits

    return DraftLM()
