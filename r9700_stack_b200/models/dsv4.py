"""DeepSeek-V4.1-Flash-class decoder: manifold hyper-connections over 4 residual
streams, sparse MLA attention with an indexer, routed experts in 3-bit trellis (EXL3-style) codes,
and Engram n-gram embeddings read from pinned host memory.

Per layer (T tokens, residual streams R [T, 4, H]):
  seam(R, previous FFN output) -> li -> RMSNorm -> MLA (+ Engram at the Engram layers) -> y_attn
  seam(R, y_attn)              -> li -> RMSNorm -> routed trellis experts + shared expert -> y_ffn
and a final seam folds the last FFN output in and collapses the streams for the head. Each seam is
one two-launch kernel pair (``ops.mhc``). Experts decode through the trellis GEMV per (expert, 16-row)
work item of the aligned routing layout, gate and up fused with SwiGLU.
Reference: r9700_vllm/models/deepseek_v41_exl3.py, r9700_vllm/models/deepseek_v41_rdna4.py:36-394,
r9700_vllm/hc_dsv4.py, r9700_vllm/quant/exl3_moe.py, r9700_vllm/moe/exl3_decode.py.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ..ops import exl3 as X
from ..ops import linear as L
from ..ops import mhc as M
from ..ops.hostmem import HostTable
from .hybrid import StepMeta
from .hybrid_moe import MoEBuffers
from .mla_moe import MLAConfig, MLAMoELM, MLAWorkspace, _ops
from .weights import WeightFactory


@dataclass
class DSV4Config(MLAConfig):
    hc: int = 4
    expert_bits: int = 3
    engram_layers: list = field(default_factory=lambda: [1])
    engram_rows: int = 1 << 22
    engram_dim: int = 512
    engram_orders: int = 2


def dsv41_flash() -> DSV4Config:
    """BASELINE config 5 (synthetic): 61 layers, hidden 7168, 128 MLA heads, 384 experts (I 2048) top-8 in
    3-bit trellis codes, 4 hyper-connection streams, Engram tables 2 x 2^22 x 512 fp8 in host memory."""
    return DSV4Config(name="dsv41-flash-exl3", hidden=7168, layers=61, vocab=129280, n_heads=128, q_lora=1536,
                      qk_nope=128, v_head=128, index_heads=64, index_topk=2048, first_dense=0, dense_ffn=18432,
                      moe_experts=384, moe_topk=8, moe_ffn=2048, moe_shared_ffn=2048, n_group=8, topk_group=4,
                      routed_scale=2.5, engram_layers=[1, 14], engram_rows=1 << 22, engram_dim=512)


def tiny_dsv4(**kw) -> DSV4Config:
    base = dict(name="tiny-dsv4", hidden=256, layers=3, vocab=512, n_heads=4, q_lora=128, qk_nope=64, v_head=64,
                index_heads=4, index_topk=24, first_dense=0, dense_ffn=512, moe_experts=8, moe_topk=2, moe_ffn=256,
                moe_shared_ffn=256, n_group=2, topk_group=1, routed_scale=1.0, engram_layers=[1],
                engram_rows=4096, engram_dim=256)
    base.update(kw)
    return DSV4Config(**base)


class DSV4Workspace(MLAWorkspace):
    def __init__(self, m: "DSV4LM", max_tokens: int, max_logit_rows: int, max_ctx: int):
        super().__init__(m, max_tokens, max_logit_rows, max_ctx)
        c, dev = m.cfg, m.device
        H = c.hidden
        self.R = torch.zeros(max_tokens, c.hc, H, dtype=torch.bfloat16, device=dev)
        self.post = [torch.zeros(max_tokens, c.hc, device=dev) for _ in range(2)]
        self.comb = [torch.zeros(max_tokens, c.hc, c.hc, device=dev) for _ in range(2)]
        self.li = torch.zeros(max_tokens, H, dtype=torch.bfloat16, device=dev)
        self.part = torch.zeros(max_tokens * (H // 64) * 25, device=dev)
        self.y2 = torch.zeros(max_tokens, H, dtype=torch.bfloat16, device=dev)
        self.sorted_x = torch.zeros(self.moe.max_rows, H, dtype=torch.bfloat16, device=dev)
        self.h_sorted = torch.zeros(self.moe.max_rows, c.moe_ffn, dtype=torch.bfloat16, device=dev)
        self.eng_ids = torch.zeros(max_tokens, c.engram_orders, dtype=torch.int64, device=dev)
        self.eng_rows = torch.zeros(max_tokens * c.engram_orders, c.engram_dim, dtype=torch.bfloat16, device=dev)
        self.eng_sum = torch.zeros(max_tokens, c.engram_dim, dtype=torch.bfloat16, device=dev)
        self.eng_gate = torch.zeros(max_tokens, 1, dtype=torch.float32, device=dev)


class DSV4LM(MLAMoELM):
    mx_experts = False

    def __init__(self, cfg: DSV4Config, par=None, device="cuda", seed: int = 0, comm=None, max_ctx: int = 32768):
        super().__init__(cfg, par, device, seed=seed, comm=comm, max_ctx=max_ctx)

    def _build(self, seed: int):
        c = self.cfg
        super()._build(seed)  # MLA attention, dense FFN, embeddings and head of the MLA model
        wf = WeightFactory(self.device, seed=seed * 1000 + 91, std=c.init_std)
        H, El, I = c.hidden, self.e_local, c.moe_ffn
        r = self.par.tp_rank

        def mhc_params(k):
            g = torch.Generator(device=self.device).manual_seed(seed * 7919 + k)
            fn = torch.randn(24, c.hc * H, generator=g, device=self.device) * (1.0 / (c.hc * H) ** 0.5)
            base = torch.randn(24, generator=g, device=self.device) * 0.1
            return M.MHCParams(fn=fn.contiguous(), scale=torch.tensor([1.0, 1.0, 1.0], device=self.device), base=base)

        for i, lay in enumerate(self.layers):
            lay["hc_attn"], lay["hc_ffn"] = mhc_params(2 * i), mhc_params(2 * i + 1)
            if "router" in lay:
                # expert e of layer i is keyed by (layer, e): rank r's slice is the TP=1 model's experts
                seed_e = seed * 100000 + i * 10
                lay["x_gate"] = X.random_linear(H, I, c.expert_bits, self.device, seed=seed_e + 1, experts=El, first=r * El)
                lay["x_up"] = X.random_linear(H, I, c.expert_bits, self.device, seed=seed_e + 2, experts=El, first=r * El)
                lay["x_down"] = X.random_linear(I, H, c.expert_bits, self.device, seed=seed_e + 3, experts=El, first=r * El)
            if i in c.engram_layers:
                lay["engram"] = HostTable.random(c.engram_rows, c.engram_dim, "fp8", seed=seed * 31 + i, std=0.02)
                lay["eng_proj"] = L.BF16Weight(wf.randn(H, c.engram_dim, dtype=torch.bfloat16))
                lay["eng_gate"] = L.BF16Weight(wf.randn(1, H, dtype=torch.bfloat16))
        self.hc_head = mhc_params(10_000)

    def weight_bytes(self) -> int:
        from .weights import weight_nbytes

        n = self.embed.numel() * 2 + weight_nbytes(self.lm_head)
        for lay in self.layers:
            for v in lay.values():
                n += v.nbytes if isinstance(v, X.Exl3Linear) else (0 if isinstance(v, HostTable) else weight_nbytes(v))
        return n

    def alloc_caches(self, num_kv_blocks: int, num_state_slots: int, kv_block: int = 64):
        super().alloc_caches(num_kv_blocks, num_state_slots, kv_block)
        self.ng_hist = torch.full((num_state_slots, 3), -1, dtype=torch.int32, device=self.device)

    def commit(self, meta, ws, acc_len) -> None:
        """After a verify pass: advance the n-gram history by the accepted tokens."""
        c = self.cfg
        _ops().ngram_ids(meta.input_ids, meta.seq_start, acc_len, meta.seq_state_slot, meta.seq_has_state,
                         self.ng_hist, c.engram_orders, c.engram_rows, True, ws.eng_ids)

    def alloc_workspace(self, max_tokens: int, max_logit_rows: int) -> DSV4Workspace:
        return DSV4Workspace(self, max_tokens, max_logit_rows, self.max_ctx)

    # --------------------------------------------------------------------------------------------
    def _engram(self, lay, meta: StepMeta, ws: DSV4Workspace, T: int) -> None:
        """y += sigmoid(h . g) * (sum over n-gram orders of table rows) @ W_e^T."""
        c, o = self.cfg, _ops()
        ids = ws.eng_ids[:T]
        o.ngram_ids(meta.input_ids, meta.seq_start, meta.seq_len, meta.seq_state_slot, meta.seq_has_state,
                    self.ng_hist, c.engram_orders, c.engram_rows, False, ids)
        rows = ws.eng_rows[: T * c.engram_orders]
        lay["engram"].gather(ids.view(-1), rows)
        torch.sum(rows.view(T, c.engram_orders, -1), dim=1, out=ws.eng_sum[:T])
        L.bf16_linear(ws.h[:T], lay["eng_gate"], out=ws.eng_gate[:T], out_dtype=torch.float32)
        L.bf16_linear(ws.eng_sum[:T], lay["eng_proj"], out=ws.y2[:T])
        ws.y[:T].add_(ws.y2[:T] * torch.sigmoid(ws.eng_gate[:T]))

    def _ffn(self, i: int, lay, ws: DSV4Workspace, T: int) -> None:
        if "router" not in lay:
            return super()._ffn(i, lay, ws, T)
        c, o, mb = self.cfg, _ops(), ws.moe
        x = ws.h[:T]
        k, El = c.moe_topk, self.e_local
        L.bf16_linear(x, lay["router"], out=mb.logits_e[:T], out_dtype=torch.float32)
        o.moe_route(mb.logits_e[:T], k, 2, lay["router_bias"], c.n_group, c.topk_group, float(c.routed_scale), True,
                    mb.ids[:T], mb.wts[:T])
        A = T * k
        o.moe_align(mb.ids[:T], self.par.tp_rank * El, El, 16, mb.perm_row[:A], mb.seg_start, mb.work, mb.work_count)
        o.moe_gather_bf16(x, k, mb.perm_row[:A], ws.sorted_x)
        nwork = min(mb.max_work, -(-A // 16) + min(El, A))
        work = mb.work[:nwork]
        lay["x_gate"].gemv(ws.sorted_x, ws.h_sorted, work=work, work_count=mb.work_count, n_items=nwork, rows=16,
                           up=lay["x_up"])
        y_sorted = mb.y_sorted
        lay["x_down"].gemv(ws.h_sorted, y_sorted, work=work, work_count=mb.work_count, n_items=nwork, rows=16)
        L.bf16_swiglu(x, lay["s_gate"], lay["s_up"], out=mb.sh_h[:T])
        L.bf16_linear(mb.sh_h[:T], lay["s_down"], out=mb.sh_out[:T])
        o.moe_combine(y_sorted, mb.perm_row[:A], mb.wts[:T], k, mb.sh_out[:T], None, ws.y[:T])
        self.comm.all_reduce_(ws.y[:T])

    def forward(self, meta: StepMeta, ws: DSV4Workspace, T: int, R: int) -> torch.Tensor:
        c, o = self.cfg, _ops()
        H = c.hidden
        # residual streams start as copies of the token embedding
        torch.index_select(self.embed, 0, meta.input_ids[:T], out=ws.resid[:T])
        ws.R[:T].copy_(ws.resid[:T, None, :].expand(T, c.hc, H))
        so = post = comb = None
        for i, lay in enumerate(self.layers):
            _, pa, ca, _ = M.seam(ws.R[:T], lay["hc_attn"], so, post, comb, R_out=ws.R[:T], post_out=ws.post[0][:T],
                                  comb_out=ws.comb[0][:T], li=ws.li[:T], part=ws.part)
            L.rmsnorm(ws.li[:T], lay["in_norm"], c.rms_eps, out=ws.h[:T])
            self._attention(i, lay, meta, ws, T)
            if "engram" in lay:
                self._engram(lay, meta, ws, T)
            ws.y2[:T].copy_(ws.y[:T])
            _, pf, cf, _ = M.seam(ws.R[:T], lay["hc_ffn"], ws.y2[:T], pa, ca, R_out=ws.R[:T], post_out=ws.post[1][:T],
                                  comb_out=ws.comb[1][:T], li=ws.li[:T], part=ws.part)
            L.rmsnorm(ws.li[:T], lay["post_norm"], c.rms_eps, out=ws.h[:T])
            self._ffn(i, lay, ws, T)
            # the next seam reads this layer's FFN mixes: keep them out of the buffers it writes
            ws.post[0][:T].copy_(pf)
            ws.comb[0][:T].copy_(cf)
            so, post, comb = ws.y[:T], ws.post[0][:T], ws.comb[0][:T]
        M.seam(ws.R[:T], self.hc_head, so, post, comb, R_out=ws.R[:T], post_out=ws.post[1][:T],
               comb_out=ws.comb[1][:T], li=ws.li[:T], part=ws.part)
        if meta.write_state:
            o.ngram_ids(meta.input_ids, meta.seq_start, meta.seq_len, meta.seq_state_slot, meta.seq_has_state,
                        self.ng_hist, c.engram_orders, c.engram_rows, True, ws.eng_ids[:T])
        L.rmsnorm(ws.li[:T], self.final_norm, c.rms_eps, out=ws.norm_out[:T])
        rows = ws.final_rows[:R]
        torch.index_select(ws.norm_out[:T], 0, meta.logits_idx[:R], out=rows)
        L.bf16_linear(rows, self.lm_head, out=ws.logits_local[:R], out_dtype=torch.float32)
        return self.comm.all_gather_lastdim(ws.logits_local[:R], out=ws.logits[:R])
