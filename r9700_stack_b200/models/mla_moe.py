"""Sparse-MLA MoE decoder (GLM-5.3-Flash / DeepSeek-V3.2 class).

Per layer: RMSNorm -> multi-head latent attention with a lightning indexer selecting the top-k
context positions per query -> RMSNorm -> FFN (dense SwiGLU in the first ``first_dense`` layers, then
routed experts with sigmoid + bias group-limited top-k routing and a shared expert).

Attention runs in the latent space ("absorbed" MLA): the latent cache row of a position is
[rmsnorm(c_kv) (512) | rope(k_pe) (64)]; a query's nope part is mapped into the latent space by W_uk
per head, so every head scores the selected rows with one 576-long dot product and the weighted sum
of latent rows is mapped back by W_uv. The indexer scores every visible position with
sum_h w_h relu(q_h . k) (fp8 keys) and keeps the top ``index_topk``.
Reference: r9700_vllm/models/glm5next.py:39-395, r9700_vllm/attn/sparse_mla.py:37-112,
r9700_vllm/attn/indexer_logits.py:21-87, kernels/r9k_sparse_mla.hip.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

from .. import _native, knobs
from ..ops import linear as L
from ..utils import status as _status
from .config import ParallelConfig
from .hybrid import NoComm, StepMeta
from .hybrid_moe import MoEBuffers, moe_ffn
from .weights import TPFactory, WeightFactory, from_float

LAT, PE, IDX = 512, 64, 128


def _ops():
    return _native.ops()


HEAD_GEMM_MIN_TOKENS = 256


def head_project(x: torch.Tensor, W: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Per-head projection out[t, h, :N] = x[t, h, :K] @ W[h]^T (W [H, N, K] bf16). Wide batches
    (prefill) run one tcgen05 GEMM per head on strided views of x and out (tokens on the MMA's M
    side); decode-sized batches run the one-launch CUDA-core ``head_gemv``."""
    T, H = x.shape[0], W.shape[0]
    N, K = W.shape[1], W.shape[2]
    if T < HEAD_GEMM_MIN_TOKENS or K % 64 or x.stride(2) != 1 or out.stride(2) != 1:
        _ops().head_gemv(x, W, out)
        return out
    for h in range(H):
        L.bf16_linear(x[:, h, :K], L.BF16Weight(W[h]), out=out[:, h, :N])
    return out


@dataclass
class MLAConfig:
    name: str = "mla-moe"
    hidden: int = 4096
    layers: int = 47
    vocab: int = 154880
    n_heads: int = 64
    q_lora: int = 1536
    qk_nope: int = 128
    v_head: int = 128
    index_heads: int = 32
    index_topk: int = 2048
    first_dense: int = 3
    dense_ffn: int = 12288
    moe_experts: int = 256
    moe_topk: int = 8
    moe_ffn: int = 1536
    moe_shared_ffn: int = 1536
    n_group: int = 8
    topk_group: int = 4
    routed_scale: float = 2.5
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    expert_format: str = "nvfp4"
    init_std: float = 0.02
    mtp_layers: int = 1

    def scaled(self, **kw) -> "MLAConfig":
        return replace(self, **kw)


def glm53_flash() -> MLAConfig:
    """47 layers, hidden 4096, 64 MLA heads, indexer 32 x 128 top-2048, 256 experts."""
    return MLAConfig(name="mla-moe-glm53-flash")


def tiny_mla(**kw) -> MLAConfig:
    base = dict(name="tiny-mla", hidden=256, layers=3, vocab=512, n_heads=4, q_lora=128, qk_nope=64, v_head=64,
                index_heads=4, index_topk=24, first_dense=1, dense_ffn=512, moe_experts=8, moe_topk=2, moe_ffn=256,
                moe_shared_ffn=256, n_group=2, topk_group=1, routed_scale=1.0)
    base.update(kw)
    return MLAConfig(**base)


class MLAWorkspace:
    def __init__(self, m: "MLAMoELM", max_tokens: int, max_logit_rows: int, max_ctx: int):
        c, dev = m.cfg, m.device
        H, nh = c.hidden, m.nh
        self.max_tokens, self.logit_rows, self.max_ctx = max_tokens, max_logit_rows, max_ctx
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.resid = torch.zeros(max_tokens, H, **bf)
        self.y = torch.zeros(max_tokens, H, **bf)
        self.h = torch.zeros(max_tokens, H, **bf)
        self.cq_raw = torch.zeros(max_tokens, c.q_lora, **bf)
        self.cq = torch.zeros(max_tokens, c.q_lora, **bf)
        self.q = torch.zeros(max_tokens, nh, c.qk_nope + PE, **bf)
        self.qfull = torch.zeros(max_tokens, nh, LAT + PE, **bf)
        self.kv_a = torch.zeros(max_tokens, LAT + PE, **bf)
        self.ik = torch.zeros(max_tokens, IDX, **bf)
        self.qi = torch.zeros(max_tokens, c.index_heads, IDX, **bf)
        self.wi = torch.zeros(max_tokens, c.index_heads, dtype=torch.float32, device=dev)
        # attention runs in token chunks of `att_chunk` (indexer scores are [chunk, max_ctx])
        self.att_chunk = min(max_tokens, 256)
        self.scores = torch.zeros(self.att_chunk, max_ctx, dtype=torch.float32, device=dev)
        self.sel = torch.zeros(self.att_chunk, c.index_topk, dtype=torch.int32, device=dev)
        self.sel_cnt = torch.zeros(self.att_chunk, dtype=torch.int32, device=dev)
        self.nsplit = 4
        self.part_o = torch.zeros(self.att_chunk * nh, self.nsplit, LAT, dtype=torch.float32, device=dev)
        self.part_ml = torch.zeros(self.att_chunk * nh, self.nsplit, 2, dtype=torch.float32, device=dev)
        self.o_lat = torch.zeros(max_tokens, nh, LAT, **bf)
        self.o = torch.zeros(max_tokens, nh, c.v_head, **bf)
        self.ffn_h = torch.zeros(max_tokens, max(m.dense_local, 1), **bf)
        self.moe = MoEBuffers(dev, max_tokens, H, c.moe_experts, c.moe_topk, m.e_local, c.moe_ffn, m.shared_local)
        self.norm_out = torch.zeros(max_tokens, H, **bf)
        self.final_rows = torch.zeros(max_logit_rows, H, **bf)
        self.logits_local = torch.zeros(max_logit_rows, m.vocab_local, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(max_logit_rows, c.vocab, dtype=torch.float32, device=dev)
        self.spec = None
        self.acc_len = torch.zeros(max_logit_rows, dtype=torch.int32, device=dev)


class MLAMoELM:
    """Heads, FFN columns and experts are sharded over ``tp_size`` ranks; the indexer and the latent
    cache are replicated (every rank needs all positions' latent rows for its heads)."""

    mx_experts = True  # routed experts as MXFP4 (subclasses with other expert formats turn this off)

    def __init__(self, cfg: MLAConfig, par: ParallelConfig | None = None, device="cuda", seed: int = 0, comm=None,
                 max_ctx: int = 32768):
        self.cfg = cfg
        self.par = par or ParallelConfig()
        self.device = torch.device(device)
        self.comm = comm or NoComm()
        tp = self.par.tp_size
        assert cfg.n_heads % tp == 0 and cfg.moe_experts % tp == 0 and cfg.vocab % tp == 0
        self.nh = cfg.n_heads // tp
        self.dense_local = cfg.dense_ffn // tp
        self.e_local = cfg.moe_experts // tp
        self.shared_local = cfg.moe_shared_ffn // tp if cfg.moe_shared_ffn else 0
        self.vocab_local = cfg.vocab // tp
        self.max_ctx = max_ctx
        self.scale = 1.0 / math.sqrt(cfg.qk_nope + PE)
        self._build(seed)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, PE, 2, dtype=torch.float64, device=self.device) / PE))
        f = torch.outer(torch.arange(max_ctx + 64, dtype=torch.float64, device=self.device), inv)
        self.cos_sin = torch.cat([f.cos(), f.sin()], -1).float().contiguous()

    # --------------------------------------------------------------------------------------------
    def _build(self, seed: int):
        c, r = self.cfg, self.par.tp_rank
        wf = WeightFactory(self.device, seed=seed * 1000 + 17, std=c.init_std)
        tpf = TPFactory(self.device, seed=seed * 1000 + 31, std=c.init_std)
        tp = self.par.tp_size
        H, nh = c.hidden, self.nh
        QH = c.qk_nope + PE
        h0 = r * nh  # first head of this rank
        bfw = lambda t: L.BF16Weight(t.to(torch.bfloat16).contiguous())  # noqa: E731
        self.embed = wf.randn(c.vocab, H, dtype=torch.bfloat16)
        self.layers = []
        for i in range(c.layers):
            lay = {
                "in_norm": wf.norm(H, False), "post_norm": wf.norm(H, False),
                "w_dq": L.BF16Weight(wf.randn(c.q_lora, H, dtype=torch.bfloat16)), "q_norm": wf.norm(c.q_lora, False),
                "w_uq": bfw(tpf.raw_rows([(c.n_heads * QH, h0 * QH, nh * QH)], c.q_lora)),
                "w_dkv": L.BF16Weight(wf.randn(LAT + PE, H, dtype=torch.bfloat16)), "kv_norm": wf.norm(LAT, False),
                "w_uk": tpf.full(c.n_heads, LAT, c.qk_nope, std=0.05)[h0:h0 + nh].to(torch.bfloat16).contiguous(),
                "w_uv": tpf.full(c.n_heads, c.v_head, LAT, std=0.05)[h0:h0 + nh].to(torch.bfloat16).contiguous(),
                "w_o": bfw(tpf.full(H, c.n_heads * c.v_head)[:, h0 * c.v_head:(h0 + nh) * c.v_head]),
                "w_iq": L.BF16Weight(wf.randn(c.index_heads * IDX, c.q_lora, dtype=torch.bfloat16)),
                "w_ik": L.BF16Weight(wf.randn(IDX, H, dtype=torch.bfloat16)), "ik_norm": wf.norm(IDX, False),
                "w_iw": L.BF16Weight(wf.randn(c.index_heads, H, dtype=torch.bfloat16)),
            }
            if i < c.first_dense:
                dl = self.dense_local
                lay["w_gate"] = bfw(tpf.raw_rows([(c.dense_ffn, r * dl, dl)], H))
                lay["w_up"] = bfw(tpf.raw_rows([(c.dense_ffn, r * dl, dl)], H))
                lay["w_down"] = bfw(tpf.full(H, c.dense_ffn)[:, r * dl:(r + 1) * dl])
            else:
                El, I, E = self.e_local, c.moe_ffn, c.moe_experts
                lay["router"] = L.BF16Weight(wf.randn(c.moe_experts, H, dtype=torch.bfloat16))
                lay["router_bias"] = (wf.randn(c.moe_experts, std=0.01)).float()
                if self.mx_experts:
                    for name, rows_per, K in (("e_gate", I, H), ("e_up", I, H), ("e_down", H, I)):
                        full = tpf.full(E * rows_per, K)
                        lay[name] = from_float(full[r * El * rows_per:(r + 1) * El * rows_per], c.expert_format,
                                               tiled=True, global_from=full)
                if self.shared_local:
                    sl, S = self.shared_local, c.moe_shared_ffn
                    lay["s_gate"] = bfw(tpf.raw_rows([(S, r * sl, sl)], H))
                    lay["s_up"] = bfw(tpf.raw_rows([(S, r * sl, sl)], H))
                    lay["s_down"] = bfw(tpf.full(H, S)[:, r * sl:(r + 1) * sl])
            self.layers.append(lay)
        self.final_norm = wf.norm(H, False)
        vl = self.vocab_local
        self.lm_head = bfw(tpf.raw_rows([(c.vocab, r * vl, vl)], H))
        self.mx = False

    def weight_bytes(self) -> int:
        from .weights import weight_nbytes

        n = self.embed.numel() * 2 + weight_nbytes(self.lm_head)
        for lay in self.layers:
            n += sum(weight_nbytes(v) for v in lay.values())
        return n

    def alloc_caches(self, num_kv_blocks: int, num_state_slots: int, kv_block: int = 64):
        assert kv_block == 64
        self.lat, self.icache = {}, {}
        for i in range(self.cfg.layers):
            self.lat[i] = torch.zeros(num_kv_blocks, 64, LAT + PE, dtype=torch.bfloat16, device=self.device)
            self.icache[i] = torch.zeros(num_kv_blocks, 64, IDX, dtype=torch.uint8, device=self.device)

    def alloc_workspace(self, max_tokens: int, max_logit_rows: int) -> MLAWorkspace:
        return MLAWorkspace(self, max_tokens, max_logit_rows, self.max_ctx)

    def alloc_spec(self, ws, max_verify_tokens: int) -> None:
        ws.spec_tokens = max_verify_tokens  # no recurrent state: verification needs no commit buffers

    def commit(self, meta, ws, acc_len) -> None:
        return None

    # --------------------------------------------------------------------------------------------
    def _attention(self, i: int, lay, meta: StepMeta, ws: MLAWorkspace, T: int) -> None:
        c, o = self.cfg, _ops()
        nh = self.nh
        h = ws.h[:T]
        L.bf16_linear(h, lay["w_dq"], out=ws.cq_raw[:T])
        L.rmsnorm(ws.cq_raw[:T], lay["q_norm"], c.rms_eps, out=ws.cq[:T])
        q = ws.q[:T]
        L.bf16_linear(ws.cq[:T], lay["w_uq"], out=q.view(T, -1))
        o.rope_heads(q, nh, c.qk_nope, meta.positions, self.cos_sin)
        qf = ws.qfull[:T]
        head_project(q[:, :, : c.qk_nope], lay["w_uk"], qf[:, :, :LAT])
        qf[:, :, LAT:].copy_(q[:, :, c.qk_nope:])
        L.bf16_linear(h, lay["w_dkv"], out=ws.kv_a[:T])
        L.bf16_linear(h, lay["w_ik"], out=ws.ik[:T])
        o.mla_cache_write(ws.kv_a[:T], lay["kv_norm"], ws.ik[:T], lay["ik_norm"], c.rms_eps, meta.positions,
                          self.cos_sin, meta.slots, self.lat[i], self.icache[i])
        L.bf16_linear(ws.cq[:T], lay["w_iq"], out=ws.qi[:T].view(T, -1))
        o.rope_heads(ws.qi[:T], c.index_heads, 0, meta.positions, self.cos_sin)
        L.bf16_linear(h, lay["w_iw"], out=ws.wi[:T], alpha=1.0 / math.sqrt(c.index_heads * IDX),
                      out_dtype=torch.float32)
        C = ws.att_chunk
        for t0 in range(0, T, C):
            n = min(C, T - t0)
            sl = slice(t0, t0 + n)
            o.indexer_score(ws.qi[sl], ws.wi[sl], self.icache[i], meta.block_table, meta.tok_seq[sl],
                            meta.tok_ctx[sl], ws.max_ctx, ws.scores[:n], _status.status(self.device))
            o.topk_select(ws.scores[:n], meta.tok_ctx[sl], c.index_topk, ws.sel[:n], ws.sel_cnt[:n])
            po = ws.part_o[: n * nh]
            pml = ws.part_ml[: n * nh]
            if knobs.get("R9K_MLA_ATTN") == "simple":
                o.sparse_mla_decode(qf[sl], self.lat[i], meta.block_table, meta.tok_seq[sl], ws.sel[:n],
                                    ws.sel_cnt[:n], self.scale, po, pml, ws.o_lat[sl])
            else:
                o.sparse_mla_decode_tc(qf[sl], self.lat[i], meta.block_table, meta.tok_seq[sl], ws.sel[:n],
                                       ws.sel_cnt[:n], self.scale, po, pml, ws.o_lat[sl], _status.status(self.device))
        head_project(ws.o_lat[:T], lay["w_uv"], ws.o[:T])
        L.bf16_linear(ws.o[:T].view(T, -1), lay["w_o"], out=ws.y[:T])
        self.comm.all_reduce_(ws.y[:T])

    def _ffn(self, i: int, lay, ws: MLAWorkspace, T: int) -> None:
        c = self.cfg
        x = ws.h[:T]
        if "w_gate" in lay:
            L.bf16_swiglu(x, lay["w_gate"], lay["w_up"], out=ws.ffn_h[:T])
            L.bf16_linear(ws.ffn_h[:T], lay["w_down"], out=ws.y[:T])
        else:
            moe_ffn(lay, x, ws.moe, ws.y[:T], k=c.moe_topk, e0=self.par.tp_rank * self.e_local, E_local=self.e_local,
                    moe_ffn=c.moe_ffn, hidden=c.hidden, shared_local=self.shared_local, route_mode=1,
                    bias=lay["router_bias"], n_group=c.n_group, topk_group=c.topk_group, scale=c.routed_scale)
        self.comm.all_reduce_(ws.y[:T])

    def forward(self, meta: StepMeta, ws: MLAWorkspace, T: int, R: int) -> torch.Tensor:
        c = self.cfg
        torch.index_select(self.embed, 0, meta.input_ids[:T], out=ws.resid[:T])
        for i, lay in enumerate(self.layers):
            if i == 0:
                L.rmsnorm(ws.resid[:T], lay["in_norm"], c.rms_eps, out=ws.h[:T])
            else:
                L.rmsnorm(ws.y[:T], lay["in_norm"], c.rms_eps, residual=ws.resid[:T], residual_out=ws.resid[:T],
                          out=ws.h[:T])
            self._attention(i, lay, meta, ws, T)
            L.rmsnorm(ws.y[:T], lay["post_norm"], c.rms_eps, residual=ws.resid[:T], residual_out=ws.resid[:T],
                      out=ws.h[:T])
            self._ffn(i, lay, ws, T)
        L.rmsnorm(ws.y[:T], self.final_norm, c.rms_eps, residual=ws.resid[:T], residual_out=ws.resid[:T],
                  out=ws.norm_out[:T])
        rows = ws.final_rows[:R]
        torch.index_select(ws.norm_out[:T], 0, meta.logits_idx[:R], out=rows)
        L.bf16_linear(rows, self.lm_head, out=ws.logits_local[:R], out_dtype=torch.float32)
        return self.comm.all_gather_lastdim(ws.logits_local[:R], out=ws.logits[:R])
