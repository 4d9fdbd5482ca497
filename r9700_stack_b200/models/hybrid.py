"""Hybrid Gated-DeltaNet / full-attention decoder on the sm_100a kernel library.

Layer pattern: three GDN layers then one gated full-attention layer (``full_attn_interval``), each
followed by a SwiGLU FFN (dense, or routed MoE in the Flash-Next class). This is the architecture
class of the reference's Qwen3.5/3.8 dense and Flash-Next models (r9700_vllm/models/qwen3_5.py,
r9700_vllm/models/qwen4_exp.py, r9700_vllm/models/gdn.py).

Tensor parallelism: heads, FFN columns and experts are sharded over ``tp_size`` ranks; the outputs of
o_proj / out_proj / down_proj are partial sums reduced by ``comm.all_reduce_`` (the fused NVLink
kernels of ``parallel`` or NCCL), and the residual add is fused into the next RMSNorm.

Every op writes into a preallocated :class:`Workspace`, so a decode step is capturable in a CUDA
graph.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import _native, knobs
from ..ops import linear as L
from .config import HybridConfig, ParallelConfig
from ..utils import status as _status
from .weights import TPFactory, WeightFactory, from_float


def _ops():
    return _native.ops()


class NoComm:
    world_size = 1
    rank = 0

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        return t

    def all_gather_lastdim(self, t: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if out is not None:
            out.copy_(t)
            return out
        return t


# ------------------------------------------------------------------------------------------------
# step metadata (device tensors; the runner fills static copies for graph replay)
# ------------------------------------------------------------------------------------------------
@dataclass
class StepMeta:
    input_ids: torch.Tensor  # [T] int32
    positions: torch.Tensor  # [T] int32
    slots: torch.Tensor  # [T] int32 KV slot (-1 = padding)
    tok_seq: torch.Tensor  # [T] int32 row in block_table
    tok_ctx: torch.Tensor  # [T] int32 attention context length (pos + 1)
    block_table: torch.Tensor  # [S, max_blocks] int32
    # GDN
    tok_state_slot: torch.Tensor  # [T] int32
    tok_pos_in_chunk: torch.Tensor  # [T] int32
    tok_has_state: torch.Tensor  # [T] int32
    seq_state_slot: torch.Tensor  # [S] int32
    seq_start: torch.Tensor  # [S] int32
    seq_len: torch.Tensor  # [S] int32
    seq_has_state: torch.Tensor  # [S] int32
    logits_idx: torch.Tensor  # [R] int32 rows of the token batch whose logits are needed
    write_state: bool = True  # False during speculative verification
    # host copy of (first token, tokens) per sequence for eager prefill steps; None on the decode path
    host_seqs: list | None = None
    # host upper bound of tok_ctx on eager steps (None in CUDA graphs): QSA runs dense below its top-k
    host_max_ctx: int | None = None
    # prefill attention tile table (built once per step on first use, shared by every attention layer)
    attn_tiles: dict | None = None
    # chunked-GDN tables of an eager prefill step (built on first use, shared by every GDN layer)
    gdn_chunks: tuple | None = None


class Workspace:
    """Persistent activation buffers for up to ``max_tokens`` tokens."""

    def __init__(self, model: "HybridLM", max_tokens: int, max_logit_rows: int):
        c, dev = model.cfg, model.device
        H = c.hidden
        self.max_tokens = max_tokens
        self.resid = torch.zeros(max_tokens, H, dtype=torch.bfloat16, device=dev)
        self.y = torch.zeros(max_tokens, H, dtype=torch.bfloat16, device=dev)  # mixer / ffn partial output
        self.norm_out = torch.zeros(max_tokens, H, dtype=torch.bfloat16, device=dev)
        self.act = L.alloc_act(max_tokens, H, dev)
        a = model.attn_dims
        self.qkv = torch.zeros(max_tokens, a["qkv_rows"], dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros(max_tokens, a["hq"], c.head_dim, dtype=torch.bfloat16, device=dev)
        self.attn_act = L.alloc_act(max_tokens, a["hq"] * c.head_dim, dev)
        self.attn_bf16 = torch.zeros(max_tokens, a["hq"] * c.head_dim, dtype=torch.bfloat16, device=dev)
        g = model.gdn_dims
        self.proj = torch.zeros(max_tokens, g["proj_rows"], dtype=torch.bfloat16, device=dev)
        self.gq = torch.zeros(max_tokens, g["hk"], c.gdn_head_dim, dtype=torch.float32, device=dev)
        self.gk = torch.zeros(max_tokens, g["hk"], c.gdn_head_dim, dtype=torch.float32, device=dev)
        self.gv = torch.zeros(max_tokens, g["hv"], c.gdn_head_dim, dtype=torch.float32, device=dev)
        self.gg = torch.zeros(max_tokens, g["hv"], dtype=torch.float32, device=dev)
        self.gb = torch.zeros(max_tokens, g["hv"], dtype=torch.float32, device=dev)
        self.go = torch.zeros(max_tokens, g["hv"], c.gdn_head_dim, dtype=torch.float32, device=dev)
        self.gdn_act = L.alloc_act(max_tokens, g["hv"] * c.gdn_head_dim, dev)
        self.gdn_bf16 = torch.zeros(max_tokens, g["hv"] * c.gdn_head_dim, dtype=torch.bfloat16, device=dev)
        if model.ffn_local > 0:
            self.ffn_act = L.alloc_act(max_tokens, model.ffn_local, dev)
            if not model.mx:
                self.ffn_bf16 = torch.zeros(max_tokens, model.ffn_local, dtype=torch.bfloat16, device=dev)
        # split-KV partials for the tcgen05 decode attention
        self.nsplit_max = 16
        rows = max_logit_rows * a["hq"]
        self.part_o = torch.zeros(rows, self.nsplit_max, c.head_dim, dtype=torch.float32, device=dev)
        self.part_ml = torch.zeros(rows, self.nsplit_max, 2, dtype=torch.float32, device=dev)
        self.logit_rows = max_logit_rows
        self.final_act = L.alloc_act(max_logit_rows, H, dev)
        self.final_bf16 = torch.zeros(max_logit_rows, H, dtype=torch.bfloat16, device=dev)
        self.logits_local = torch.zeros(max_logit_rows, model.vocab_local, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(max_logit_rows, c.vocab, dtype=torch.float32, device=dev)
        if c.qsa_topk:
            self.qsa_proj = torch.zeros(max_tokens, (c.qsa_heads + 1) * 128, dtype=torch.bfloat16, device=dev)
            self.qsa_w = torch.full((max_tokens, c.qsa_heads), 128 ** -0.5, dtype=torch.float32, device=dev)
            self.qsa_vis = torch.zeros(max_tokens, dtype=torch.int32, device=dev)
            self.qsa_sel = torch.zeros(max_tokens, c.qsa_topk, dtype=torch.int32, device=dev)
            self.qsa_cnt = torch.zeros(max_tokens, dtype=torch.int32, device=dev)
            # indexer scores, viewed as [rows, groups] per call (rows chunked to fit): one fixed buffer,
            # since captured decode graphs keep the address they saw
            self.qsa_scores = torch.empty(16 << 20, dtype=torch.float32, device=dev)
        if c.hc_streams:
            HC = c.hc_streams
            self.hc_x = torch.zeros(max_tokens, HC * H, dtype=torch.bfloat16, device=dev)  # residual streams
            self.hc_n = torch.zeros(max_tokens, HC * H, dtype=torch.bfloat16, device=dev)  # normalised streams
            self.hc_l = torch.zeros(max_tokens, HC, dtype=torch.float32, device=dev)
        self.spec = None  # per-GDN-layer verify buffers (alloc_spec)
        self.spec_table = None
        self.acc_len = torch.zeros(max_logit_rows, dtype=torch.int32, device=dev)


class HybridLM:
    def __init__(self, cfg: HybridConfig, par: ParallelConfig | None = None, device="cuda", seed: int = 0,
                 comm=None):
        self.cfg = cfg
        self.par = par or ParallelConfig()
        self.device = torch.device(device)
        self.comm = comm or NoComm()
        tp, r = self.par.tp_size, self.par.tp_rank
        c = cfg
        assert c.n_q_heads % tp == 0 and c.gdn_v_heads % tp == 0 and c.gdn_k_heads % tp == 0
        hq = c.n_q_heads // tp
        hkv = max(1, c.n_kv_heads // tp)  # kv heads replicate when tp > n_kv_heads
        self.attn_dims = dict(hq=hq, hkv=hkv, qkv_rows=(2 * hq if c.attn_output_gate else hq) * c.head_dim + 2 * hkv * c.head_dim)
        hk, hv, d = c.gdn_k_heads // tp, c.gdn_v_heads // tp, c.gdn_head_dim
        self.gdn_dims = dict(hk=hk, hv=hv, conv_ch=2 * hk * d + hv * d, proj_rows=2 * hk * d + 2 * hv * d + 2 * hv)
        self.ffn_local = c.ffn // tp if c.ffn else 0
        assert c.vocab % tp == 0
        self.vocab_local = c.vocab // tp
        self.sm_scale = 1.0 / math.sqrt(c.head_dim)
        self.k_scale = 1.0
        self.v_scale = 1.0
        self._build(seed)
        self._rope_cache(8192 * 8)
        self.trace = None  # utils.trace.DeviceTrace: %globaltimer marks between sublayers

    # --------------------------------------------------------------------------------------------
    def _build(self, seed: int):
        c, tp, r = self.cfg, self.par.tp_size, self.par.tp_rank
        wf = WeightFactory(self.device, seed=seed * 1000 + 17, std=c.init_std)
        fmt = c.weight_format
        H = c.hidden
        # embeddings replicated on every rank (HBM is plentiful; saves an all-reduce per step)
        self.embed = wf.randn(c.vocab, H, std=c.init_std, dtype=torch.bfloat16)
        self.layers = []
        a, g = self.attn_dims, self.gdn_dims
        # sharded tensors: the whole model's tensor from its own seed, cut to this rank's shard
        tpf = TPFactory(self.device, seed=seed * 1000 + 31, std=c.init_std)
        D, d = c.head_dim, c.gdn_head_dim
        hq, hkv = a["hq"], a["hkv"]
        kv0 = (r * hq) // (c.n_q_heads // c.n_kv_heads)  # first kv head of this rank (replicated past tp = n_kv)
        qseg = (c.n_q_heads * D, r * hq * D, hq * D)
        kvseg = (c.n_kv_heads * D, kv0 * D, hkv * D)
        qkv_segs = [qseg, qseg, kvseg, kvseg] if c.attn_output_gate else [qseg, kvseg, kvseg]
        hk, hv = g["hk"], g["hv"]
        kseg = (c.gdn_k_heads * d, r * hk * d, hk * d)
        vseg = (c.gdn_v_heads * d, r * hv * d, hv * d)
        hseg = (c.gdn_v_heads, r * hv, hv)
        for i in range(c.layers):
            lay = {"attn": c.is_attention(i)}
            lay["in_norm"] = wf.norm(H, c.norm_plus_one)
            lay["post_norm"] = wf.norm(H, c.norm_plus_one)
            if lay["attn"]:
                lay["w_qkv"] = tpf.rows(qkv_segs, H, fmt)
                lay["w_o"] = tpf.cols(H, c.n_q_heads * D, r * hq * D, hq * D, fmt)
                lay["q_norm"] = wf.norm(c.head_dim, c.norm_plus_one)
                lay["k_norm"] = wf.norm(c.head_dim, c.norm_plus_one)
                if c.qsa_topk:
                    # indexer (replicated on every rank so all ranks select the same groups):
                    # qsa_heads query heads + one key head of 128, one shared norm, rope on dims [0, 64)
                    lay["w_idx"] = wf.linear((c.qsa_heads + 1) * 128, H, fmt)
                    lay["idx_norm"] = wf.norm(128, c.norm_plus_one)
            else:
                # in_proj rows: [q | k | v | z | b | a], each split by heads
                lay["w_in"] = tpf.rows([kseg, kseg, vseg, vseg, hseg, hseg], H, fmt)
                lay["w_out"] = tpf.cols(H, c.gdn_v_heads * d, r * hv * d, hv * d, fmt)
                lay["conv_w"] = tpf.raw_rows([kseg, kseg, vseg], c.conv_width, std=0.3, dtype=torch.bfloat16)
                u = torch.rand(c.gdn_v_heads, generator=tpf._gen(), device=self.device)
                lay["A_log"] = torch.log(1.0 + 15.0 * u[r * hv:(r + 1) * hv])
                lay["dt_bias"] = tpf.raw_rows([hseg], std=0.5)
                lay["gdn_norm"] = (1.0 + wf.randn(d, std=0.1)).to(torch.bfloat16)
            if c.hc_streams:
                from ..ops import hc as HCo

                lay["hc_in"] = HCo.random_point(wf, c.hc_streams, H)
                lay["hc_post"] = HCo.random_point(wf, c.hc_streams, H)
            if self.ffn_local:
                fl = self.ffn_local
                lay["w_gate"] = tpf.rows([(c.ffn, r * fl, fl)], H, fmt)
                lay["w_up"] = tpf.rows([(c.ffn, r * fl, fl)], H, fmt)
                lay["w_down"] = tpf.cols(H, c.ffn, r * fl, fl, fmt)
            self.layers.append(lay)
        self.final_norm = wf.norm(H, c.norm_plus_one)
        if c.hc_streams:
            from ..ops import hc as HCo

            self.hc_final = HCo.random_point(wf, c.hc_streams, H)
        vl = self.vocab_local
        self.lm_head = tpf.rows([(c.vocab, r * vl, vl)], H, c.lm_head_format)
        # MX weights take MXFP8 activations; bf16 and native NVFP4 weights take bf16 activations
        kinds = {isinstance(w, L.MXWeight) for lay in self.layers for n, w in lay.items()
                 if n in ("w_in", "w_out", "w_qkv", "w_o", "w_idx", "w_gate", "w_up", "w_down")}
        assert len(kinds) == 1, "every layer's linear weights must be MX, or all bf16 / native NVFP4"
        self.mx = kinds.pop()

    def _rope_cache(self, max_pos: int):
        c = self.cfg
        rot = c.rotary_dim
        inv = 1.0 / (c.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float64, device=self.device) / rot))
        t = torch.arange(max_pos, dtype=torch.float64, device=self.device)
        f = torch.outer(t, inv)
        self.cos_sin = torch.cat([f.cos(), f.sin()], dim=-1).float().contiguous()

    # --------------------------------------------------------------------------------------------
    def weight_bytes(self) -> int:
        from .weights import weight_nbytes

        n = self.embed.numel() * 2 + weight_nbytes(self.lm_head)
        for lay in self.layers:
            for v in lay.values():
                n += weight_nbytes(v)
        return n

    def alloc_workspace(self, max_tokens: int, max_logit_rows: int) -> Workspace:
        return Workspace(self, max_tokens, max_logit_rows)

    def alloc_caches(self, num_kv_blocks: int, num_state_slots: int, kv_block: int = 64):
        c, a, g = self.cfg, self.attn_dims, self.gdn_dims
        kv = {}
        for i in c.attn_layers:
            kv[i] = (
                torch.zeros(num_kv_blocks, a["hkv"], kv_block, c.head_dim, dtype=torch.uint8, device=self.device),
                torch.zeros(num_kv_blocks, a["hkv"], kv_block, c.head_dim, dtype=torch.uint8, device=self.device),
            )
        sdt = torch.float32 if c.gdn_state_dtype == "fp32" else torch.bfloat16
        ssm, conv = {}, {}
        for i in c.gdn_layers:
            ssm[i] = torch.zeros(num_state_slots, g["hv"], c.gdn_head_dim, c.gdn_head_dim, dtype=sdt, device=self.device)
            conv[i] = torch.zeros(num_state_slots, g["conv_ch"], c.conv_width - 1, dtype=sdt, device=self.device)
        self.kv, self.ssm, self.conv = kv, ssm, conv
        # QSA: token indexer keys (bf16) and mean-pooled group keys (e4m3), paged like the KV cache
        self.qsa_cache = {}
        if c.qsa_topk:
            for i in c.attn_layers:
                self.qsa_cache[i] = (
                    torch.zeros(num_kv_blocks, kv_block, 128, dtype=torch.bfloat16, device=self.device),
                    torch.zeros(num_kv_blocks, kv_block, 128, dtype=torch.uint8, device=self.device),
                )

    def alloc_spec(self, ws: Workspace, max_verify_tokens: int) -> None:
        """Per-GDN-layer buffers a verify pass fills (projections and the conv/recurrence inputs of
        every verified token), from which :meth:`commit` replays the accepted tokens, plus the
        device table of their addresses that the one-launch commit kernel reads."""
        c, g, dev = self.cfg, self.gdn_dims, self.device
        Tv, d = max_verify_tokens, c.gdn_head_dim
        ws.spec, rows = {}, []
        for i in c.gdn_layers:
            b = dict(
                proj=torch.zeros(Tv, g["proj_rows"], dtype=torch.bfloat16, device=dev),
                k=torch.zeros(Tv, g["hk"], d, dtype=torch.float32, device=dev),
                v=torch.zeros(Tv, g["hv"], d, dtype=torch.float32, device=dev),
                g=torch.zeros(Tv, g["hv"], dtype=torch.float32, device=dev),
                b=torch.zeros(Tv, g["hv"], dtype=torch.float32, device=dev),
            )
            ws.spec[i] = b
            rows.append([b["k"].data_ptr(), b["v"].data_ptr(), b["g"].data_ptr(), b["b"].data_ptr(),
                         b["proj"].data_ptr(), self.ssm[i].data_ptr(), self.conv[i].data_ptr(), 0])
        ws.spec_table = torch.tensor(rows, dtype=torch.int64).reshape(-1, 8).to(dev)
        ws.spec_tokens = Tv

    def commit(self, meta: StepMeta, ws: Workspace, acc_len: torch.Tensor) -> None:
        """Fold the first acc_len[s] verified tokens of every sequence into its GDN state (conv and
        recurrent), all layers in one launch. Attention needs nothing: the verify pass wrote every
        verified token's KV, and positions past the accepted length are rewritten before use."""
        if not self.cfg.gdn_layers:
            return
        c, g = self.cfg, self.gdn_dims
        _ops().gdn_spec_commit(ws.spec_table, g["hk"], g["hv"], c.gdn_head_dim, g["conv_ch"], c.conv_width,
                               g["proj_rows"], self.ssm[c.gdn_layers[0]].dtype == torch.float32,
                               meta.seq_state_slot, meta.seq_start, acc_len, meta.seq_has_state)

    # --------------------------------------------------------------------------------------------
    def _linear(self, act: L.MXAct, xb: torch.Tensor, w, out: torch.Tensor):
        if isinstance(w, L.MXWeight):
            L.mx_linear(act, w, out=out)
        elif isinstance(w, L.NVF4Weight):
            L.nvf4_linear(xb, w, out=out)
        else:
            L.bf16_linear(xb, w, out=out)

    def _norm(self, x, w, ws: Workspace, T: int, residual: bool):
        """(residual add) + RMSNorm, producing MXFP8 (MX weights) or bf16 (bf16 weights) input."""
        c = self.cfg
        L.rmsnorm(
            x[:T], w, c.rms_eps, plus_one=c.norm_plus_one,
            residual=ws.resid[:T] if residual else None,
            residual_out=ws.resid[:T] if residual else None,
            out=None if self.mx else ws.norm_out[:T],
            quant_out=ws.act.narrow(T) if self.mx else None,
        )

    def _attention(self, i: int, lay, meta: StepMeta, ws: Workspace, T: int):
        c, a = self.cfg, self.attn_dims
        hq, hkv, D = a["hq"], a["hkv"], c.head_dim
        qkv = ws.qkv[:T]
        self._linear(ws.act.narrow(T), ws.norm_out[:T], lay["w_qkv"], qkv)
        gate_off = hq * D if c.attn_output_gate else -1
        k_off = (2 * hq if c.attn_output_gate else hq) * D
        v_off = k_off + hkv * D
        kc, vc = self.kv[i]
        _ops().qk_norm_rope_cache(qkv, hq, hkv, 0, k_off, v_off, lay["q_norm"], lay["k_norm"], c.rms_eps,
                                  c.norm_plus_one, meta.positions, self.cos_sin, c.rotary_dim, meta.slots,
                                  ws.q[:T], kc, vc, self.k_scale, self.v_scale)
        gate = qkv[:, gate_off:gate_off + hq * D] if gate_off >= 0 else None
        if c.qsa_topk and self._qsa(i, lay, meta, ws, T, gate):
            if self.mx:
                L.quant_act(ws.attn_bf16[:T], out=ws.attn_act.narrow(T))
            return ws.attn_act.narrow(T), ws.attn_bf16[:T], lay["w_o"]
        out_q = ws.attn_act.q[:T] if self.mx else None
        out_sf = ws.attn_act.sf if self.mx else None
        out_bf = None if self.mx else ws.attn_bf16[:T]
        G = hq // hkv
        if knobs.get("R9K_ATTN") == "simple" or D != 256:
            _ops().paged_attention(ws.q[:T], kc, vc, meta.block_table, meta.tok_seq, meta.tok_ctx, self.sm_scale,
                                   self.k_scale, self.v_scale, gate, out_bf, out_q, out_sf, 0)
        elif meta.host_seqs is not None and (T > ws.logit_rows or any(n * G > 128 for _, n in meta.host_seqs)):
            # prefill: query tiles of floor(128 / G) tokens, whole causal key range per CTA
            tt = self._attn_tile_table(meta, 128 // G)
            _ops().attn_tc_prefill(ws.q[:T], kc, vc, meta.block_table, meta.tok_ctx, tt, tt.shape[0] // 3,
                                   self.sm_scale, self.k_scale, self.v_scale, gate, out_bf, out_q, out_sf,
                                   _status.status(self.device))
        else:
            S = meta.seq_start.shape[0]
            max_rows = max(n for _, n in meta.host_seqs) if meta.host_seqs else 1
            if max_rows * G <= 16:
                # keys-on-M decode kernel: one CTA per SM, so one wave of splits over the 148 SMs
                nsplit = max(1, min(ws.nsplit_max, 148 // (S * hkv)))
            else:
                nsplit = max(1, min(ws.nsplit_max, -(-296 // (S * hkv))))
            po = ws.part_o.view(-1)[: T * hq * nsplit * D].view(T * hq, nsplit, D)
            pml = ws.part_ml.view(-1)[: T * hq * nsplit * 2].view(T * hq, nsplit, 2)
            _ops().attn_tc_decode(ws.q[:T], kc, vc, meta.block_table, meta.tok_ctx, meta.seq_start, meta.seq_len,
                                  self.sm_scale, self.k_scale, self.v_scale, po, pml, gate, out_bf, out_q, out_sf,
                                  _status.status(self.device), max_rows)
        return ws.attn_act.narrow(T), ws.attn_bf16[:T], lay["w_o"]

    def _attn_tile_table(self, meta: StepMeta, qt: int) -> torch.Tensor:
        """(sequence, first token, rows) per prefill query tile of qt tokens: built once per step from
        the host sequence list and uploaded from pinned memory, then reused by every attention layer."""
        # step metadata views are reused across steps of the same shape: the table belongs to this
        # step's host sequence list (held by the cache, so an identity check cannot be fooled)
        if meta.attn_tiles is None or meta.attn_tiles.get("seqs") is not meta.host_seqs:
            meta.attn_tiles = {"seqs": meta.host_seqs}
        tt = meta.attn_tiles.get(qt)
        if tt is None:
            import numpy as np

            rows = []
            for si, (t0, n) in enumerate(meta.host_seqs):
                j = np.arange(0, n, qt, dtype=np.int32)
                rows.append(np.stack([np.full_like(j, si), t0 + j, np.minimum(qt, n - j)], axis=1))
            host = torch.from_numpy(np.concatenate(rows).reshape(-1)).pin_memory()
            tt = host.to(self.device, non_blocking=True)
            meta.attn_tiles[qt] = tt
        return tt

    def _qsa(self, i: int, lay, meta: StepMeta, ws: Workspace, T: int, gate) -> bool:
        """QSA indexer for attention layer i (projection, norm + rope, token key store, group
        compression) and, unless every row's context fits inside the top-k (then the selection is the
        whole causal context and the dense kernels run), scoring, top-k and the sparse attention into
        ws.attn_bf16. Returns True when the sparse attention ran."""
        c, a = self.cfg, self.attn_dims
        Hi, k = c.qsa_heads, c.qsa_topk
        o = _ops()
        proj = ws.qsa_proj[:T]
        self._linear(ws.act.narrow(T), ws.norm_out[:T], lay["w_idx"], proj)
        heads = proj.view(T * (Hi + 1), 128)
        L.rmsnorm(heads, lay["idx_norm"], c.rms_eps, plus_one=c.norm_plus_one, out=heads)
        o.rope_heads(proj.view(T, Hi + 1, 128), Hi + 1, 0, meta.positions, self.cos_sin)
        ktok, ckey = self.qsa_cache[i]
        o.qsa_key_write(proj[:, Hi * 128:], meta.slots, ktok)
        o.qsa_compress(ktok, meta.block_table, meta.tok_seq, meta.tok_ctx, ckey)
        if meta.host_max_ctx is not None and meta.host_max_ctx <= 4 * k + 3:
            return False
        vis = ws.qsa_vis[:T]
        torch.floor_divide(meta.tok_ctx[:T], 4, out=vis)
        groups = meta.block_table.shape[1] * 16
        rows = min(T, ws.qsa_scores.numel() // groups)
        assert rows >= 1, "context too long for the QSA score buffer"
        iq = proj[:, : Hi * 128].view(T, Hi, 128)
        for r0 in range(0, T, rows):
            r1 = min(T, r0 + rows)
            sc = ws.qsa_scores[: (r1 - r0) * groups].view(r1 - r0, groups)
            o.indexer_score(iq[r0:r1], ws.qsa_w[r0:r1], ckey, meta.block_table, meta.tok_seq[r0:r1], vis[r0:r1],
                            groups, sc, _status.status(self.device))
            o.topk_select(sc, vis[r0:r1], k, ws.qsa_sel[r0:r1], ws.qsa_cnt[r0:r1])
        kc, vc = self.kv[i]
        hq, hkv = a["hq"], a["hkv"]
        nsplit = 1 if T * hkv >= 148 or T > ws.logit_rows else max(1, min(ws.nsplit_max, -(-296 // (T * hkv))))
        o.qsa_attention(ws.q[:T], kc, vc, meta.block_table, meta.tok_seq, meta.tok_ctx, ws.qsa_sel[:T],
                        ws.qsa_cnt[:T], self.sm_scale, self.k_scale, self.v_scale, nsplit, ws.part_o, ws.part_ml,
                        gate, ws.attn_bf16[:T])
        return True

    def _gdn(self, i: int, lay, meta: StepMeta, ws: Workspace, T: int):
        c, g = self.cfg, self.gdn_dims
        hk, hv, d = g["hk"], g["hv"], c.gdn_head_dim
        sb = None
        if not meta.write_state and ws.spec is not None:
            # speculative verify: keep this layer's projections and recurrence inputs for commit()
            assert T <= ws.spec_tokens, "verify batch exceeds the speculative buffers"
            sb = ws.spec[i]
        proj = (sb["proj"] if sb is not None else ws.proj)[:T]
        ssm, conv = self.ssm[i], self.conv[i]
        o = _ops()
        decode = meta.write_state and T == meta.seq_start.shape[0] and knobs.get("R9K_GDN_FUSED") != "0"
        if decode and knobs.get("R9K_GDN_PREFETCH") != "0":
            # the state rows this step updates land in L2 while in_proj streams its weights
            o.gdn_state_prefetch(ssm, conv, meta.seq_state_slot)
        self._linear(ws.act.narrow(T), ws.norm_out[:T], lay["w_in"], proj)
        z_off = 2 * hk * d + hv * d
        b_off = z_off + hv * d
        a_off = b_off + hv
        if decode:
            # decode: every sequence has one token -> one fused kernel per layer
            o.gdn_decode_fused(proj, hk, hv, z_off, b_off, a_off, lay["conv_w"], conv, ssm, meta.seq_state_slot,
                               meta.seq_has_state, lay["A_log"], lay["dt_bias"], lay["gdn_norm"], c.rms_eps,
                               ws.gdn_act.q[:T] if self.mx else None, ws.gdn_act.sf if self.mx else None,
                               None if self.mx else ws.gdn_bf16[:T])
            return ws.gdn_act.narrow(T), ws.gdn_bf16[:T], lay["w_out"]
        gk, gv, gg, gb = (ws.gk, ws.gv, ws.gg, ws.gb) if sb is None else (sb["k"], sb["v"], sb["g"], sb["b"])
        # long prefill: the chunked delta rule on the tensor cores (same state and output)
        chunked = (sb is None and meta.write_state and bool(meta.host_seqs)
                   and knobs.get("R9K_GDN_PREFILL") == "chunked"
                   and max(n for _, n in meta.host_seqs) >= knobs.get_int("R9K_GDN_CHUNK_MIN"))
        ctab = c0 = buf = None
        if chunked:
            ctab, c0, nch = self._gdn_chunk_tables(meta)
            buf = self._gdn_chunk_scratch(ws, nch * hv * 128, T * (2 * hk + hv) * 128)
        o.gdn_conv_prep(proj, hk, hv, d, d, b_off, a_off, lay["conv_w"], conv, meta.tok_state_slot,
                        meta.tok_pos_in_chunk, meta.tok_has_state, lay["A_log"], lay["dt_bias"],
                        ws.gq[:T], gk[:T], gv[:T], gg[:T], gb[:T], buf[0] if chunked else None)
        if meta.write_state:
            o.gdn_conv_state_update(proj, conv, meta.seq_state_slot, meta.seq_start, meta.seq_len, meta.seq_has_state)
        if chunked:
            o.gdn_chunked(buf[0], gg[:T], gb[:T], ssm, ctab, c0, meta.seq_state_slot, meta.seq_has_state, True, hk, hv,
                          *buf[1:], ws.go[:T], _status.status(self.device))
        else:
            o.gdn_recurrent(ws.gq[:T], gk[:T], gv[:T], gg[:T], gb[:T], ssm, meta.seq_state_slot,
                            meta.seq_start, meta.seq_len, meta.seq_has_state, meta.write_state, ws.go[:T])
        if self.mx:
            o.gdn_out_norm_quant(ws.go[:T], proj, z_off, lay["gdn_norm"], c.rms_eps, None, ws.gdn_act.q[:T],
                                 ws.gdn_act.sf)
        else:
            o.gdn_out_norm_quant(ws.go[:T], proj, z_off, lay["gdn_norm"], c.rms_eps, ws.gdn_bf16[:T], None, None)
        return ws.gdn_act.narrow(T), ws.gdn_bf16[:T], lay["w_out"]

    def _gdn_chunk_tables(self, meta: StepMeta):
        """(chunk table [chunks, 3] = first token, tokens, sequence; first chunk of each sequence [S + 1];
        chunk count) for the chunked GDN prefill, 128 tokens per chunk, built once per step."""
        if meta.gdn_chunks is not None and meta.gdn_chunks[0] is meta.host_seqs:
            return meta.gdn_chunks[1:]
        rows, first = [], [0]
        for si, (t0, n) in enumerate(meta.host_seqs):
            rows += [(t0 + j, min(128, n - j), si) for j in range(0, n, 128)]
            first.append(len(rows))
        host = torch.tensor(rows or [(0, 0, 0)], dtype=torch.int32).reshape(-1).pin_memory()
        hf = torch.tensor(first, dtype=torch.int32).pin_memory()
        ctab = host.to(self.device, non_blocking=True).view(-1, 3)[: len(rows)]
        c0 = hf.to(self.device, non_blocking=True)
        meta.gdn_chunks = (meta.host_seqs, ctab, c0, len(rows))
        return ctab, c0, len(rows)

    def _gdn_chunk_scratch(self, ws: Workspace, rows: int, qkv_elems: int):
        """Buffers of the chunked GDN: the bf16 q|k|v copy of the conv step, then phase 1's outputs (W,
        gamma q, K-hat, P in bf16; U^T fp32; gamma_C), grown on demand (eager prefill steps only)."""
        buf = getattr(ws, "gdn_chunk_buf", None)
        if buf is None or buf[1].shape[0] < rows or buf[0].numel() < qkv_elems:
            cap = max(rows, 128 * 16, buf[1].shape[0] if buf is not None else 0)
            qcap = max(qkv_elems, buf[0].numel() if buf is not None else 0)
            dev = self.device
            bf = lambda: torch.empty(cap, 128, dtype=torch.bfloat16, device=dev)
            buf = (torch.empty(qcap, dtype=torch.bfloat16, device=dev), bf(), bf(), bf(), bf(),
                   torch.empty(cap, 128, dtype=torch.float32, device=dev),
                   torch.empty(cap // 128, dtype=torch.float32, device=dev))
            ws.gdn_chunk_buf = buf
        return buf

    def _ffn(self, lay, ws: Workspace, T: int):
        """Gate/up + SwiGLU (fused); returns the down projection's input and weight."""
        if self.mx:
            L.mx_swiglu(ws.act.narrow(T), lay["w_gate"], lay["w_up"], out=ws.ffn_act.narrow(T))
            return ws.ffn_act.narrow(T), None, lay["w_down"]
        if isinstance(lay["w_gate"], L.NVF4Weight):
            L.nvf4_swiglu(ws.norm_out[:T], lay["w_gate"], lay["w_up"], out=ws.ffn_bf16[:T])
        else:
            L.bf16_swiglu(ws.norm_out[:T], lay["w_gate"], lay["w_up"], out=ws.ffn_bf16[:T])
        return None, ws.ffn_bf16[:T], lay["w_down"]

    def _ffn_block(self, i: int, lay, meta, ws: Workspace, T: int, call: int, fused: bool) -> None:
        """The FFN sublayer including its row-parallel reduction (overridden by the MoE model)."""
        act, xb, w = self._ffn(lay, ws, T)
        self._row_parallel(act, xb, w, ws, T, call=call, fused=fused)

    def _reduce_target(self, ws: Workspace, T: int, call: int, fused: bool) -> torch.Tensor:
        """Where a sublayer writes its partial sum: this rank's symmetric buffer (pull) or ws.y."""
        if fused and self.comm.mode == "pull":
            return self.comm.out_buffer(call, T)
        return ws.y[:T]

    def _after_partial(self, ws: Workspace, T: int, call: int, fused: bool) -> None:
        """Complete the reduction of a partial written to _reduce_target()."""
        if fused and self.comm.mode == "pull":
            return
        if fused:
            self.comm.push(ws.y[:T], call)
        else:
            self.comm.all_reduce_(ws.y[:T])

    def _row_parallel(self, act, xb, w, ws: Workspace, T: int, call: int, fused: bool) -> None:
        """Output projection of a sublayer: partial sums pushed to every rank (fused) or written to
        ws.y and all-reduced by NCCL."""
        if fused and self.comm.mode == "pull":
            # partial written into this rank's symmetric buffer; the next norm pulls and reduces
            self._linear(act, xb, w, self.comm.out_buffer(call, T))
            return
        if fused and isinstance(w, L.MXWeight):
            self.comm.gemm_push(act, w, call)
            return
        self._linear(act, xb, w, ws.y[:T])
        if fused:
            self.comm.push(ws.y[:T], call)
        else:
            self.comm.all_reduce_(ws.y[:T])

    def _post_reduce_norm(self, w, ws: Workspace, T: int, call: int, fused: bool, first: bool = False,
                          final: bool = False) -> None:
        """Reduce the previous sublayer's output (fused path) + residual add + RMSNorm."""
        c = self.cfg
        if fused:
            self.comm.ar_rmsnorm(call, T, w, c.rms_eps, c.norm_plus_one, residual=ws.resid[:T],
                                 residual_out=ws.resid[:T],
                                 y=ws.norm_out[:T] if (final or not self.mx) else None,
                                 quant_out=None if (final or not self.mx) else ws.act.narrow(T))
        elif final:
            L.rmsnorm(ws.y[:T], w, c.rms_eps, plus_one=c.norm_plus_one, residual=ws.resid[:T],
                      residual_out=ws.resid[:T], out=ws.norm_out[:T])
        else:
            self._norm(ws.y, w, ws, T, residual=True)

    def _embed(self, meta: StepMeta, ws: Workspace, T: int) -> None:
        """Input of the first layer into ws.resid (token embeddings; drafters override this)."""
        torch.index_select(self.embed, 0, meta.input_ids[:T], out=ws.resid[:T])

    def forward(self, meta: StepMeta, ws: Workspace, T: int, R: int) -> torch.Tensor:
        """Run T tokens; returns fp32 logits [R, vocab] for the rows in meta.logits_idx[:R]."""
        c = self.cfg
        if c.hc_streams:
            return self._forward_hc(meta, ws, T, R)
        fused = getattr(self.comm, "fused", False) and self.comm.can_fuse(T) and knobs.get("R9K_COMM") != "nccl"
        tr = self.trace
        if tr is not None:
            tr.begin()
            tr.mark("start")
        if fused:
            self.comm.step_begin()
        self._embed(meta, ws, T)
        nl = len(self.layers)
        for i, lay in enumerate(self.layers):
            if i == 0:
                self._norm(ws.resid, lay["in_norm"], ws, T, residual=False)
            else:
                self._post_reduce_norm(lay["in_norm"], ws, T, call=2 * i - 1, fused=fused)
            if lay["attn"]:
                act, xb, w = self._attention(i, lay, meta, ws, T)
            else:
                act, xb, w = self._gdn(i, lay, meta, ws, T)
            self._row_parallel(act, xb, w, ws, T, call=2 * i, fused=fused)
            if tr is not None:
                tr.mark(f"L{i}.{'attn' if lay['attn'] else 'gdn'}")
            self._post_reduce_norm(lay["post_norm"], ws, T, call=2 * i, fused=fused)
            self._ffn_block(i, lay, meta, ws, T, call=2 * i + 1, fused=fused)
            if tr is not None:
                tr.mark(f"L{i}.ffn")
        # final: residual add + norm, then the rows that need logits
        self._post_reduce_norm(self.final_norm, ws, T, call=2 * nl - 1, fused=fused, final=True)
        out = self._lm_head(meta, ws, T, R)
        if tr is not None:
            tr.mark("lm_head")
        return out

    def _hc_point(self, p, ws: Workspace, T: int, block: bool, final: bool = False) -> None:
        """Hyper-connection norm point: inject the block output ws.y into every residual stream, normalise
        each stream, and mix the streams into the next block's input (ws.norm_out, + MXFP8 for MX weights)."""
        from ..ops import hc as HCo

        c = self.cfg
        HC = c.hc_streams
        if knobs.get("R9K_HC_FUSED") != "0":
            HCo.point(ws.hc_x[:T], ws.y[:T] if block else None, p, HC, c.rms_eps, ws.norm_out[:T])
            if self.mx and not final:
                L.quant_act(ws.norm_out[:T], out=ws.act.narrow(T))
            return
        if block:
            L.bf16_linear(ws.y[:T], p.wl, out=ws.hc_l[:T], out_dtype=torch.float32)
        HCo.combine_norm(ws.hc_x[:T], ws.y[:T] if block else None, ws.hc_l[:T] if block else None, p.w, HC, c.rms_eps,
                         ws.hc_n[:T])
        HCo.gate_mix(ws.hc_n[:T], p.g, HC, ws.norm_out[:T])
        if self.mx and not final:
            L.quant_act(ws.norm_out[:T], out=ws.act.narrow(T))

    def _forward_hc(self, meta: StepMeta, ws: Workspace, T: int, R: int) -> torch.Tensor:
        """Forward with hyper-connection residual streams (unfused all-reduce after each block)."""
        c = self.cfg
        HC, H = c.hc_streams, c.hidden
        tr = self.trace
        if tr is not None:
            tr.begin()
            tr.mark("start")
        self._embed(meta, ws, T)
        ws.hc_x[:T].view(T, HC, H).copy_(ws.resid[:T, None, :])
        for i, lay in enumerate(self.layers):
            self._hc_point(lay["hc_in"], ws, T, block=i > 0)
            if tr is not None:
                tr.mark(f"L{i}.hc")
            if lay["attn"]:
                act, xb, w = self._attention(i, lay, meta, ws, T)
            else:
                act, xb, w = self._gdn(i, lay, meta, ws, T)
            self._row_parallel(act, xb, w, ws, T, call=2 * i, fused=False)
            if tr is not None:
                tr.mark(f"L{i}.{'attn' if lay['attn'] else 'gdn'}")
            self._hc_point(lay["hc_post"], ws, T, block=True)
            if tr is not None:
                tr.mark(f"L{i}.hc")
            self._ffn_block(i, lay, meta, ws, T, call=2 * i + 1, fused=False)
            if tr is not None:
                tr.mark(f"L{i}.ffn")
        self._hc_point(self.hc_final, ws, T, block=True, final=True)
        # the stream mean stands for the pre-norm hidden state (what MTP / block drafters read)
        torch.mean(ws.hc_x[:T].view(T, HC, H), dim=1, out=ws.resid[:T])
        out = self._lm_head(meta, ws, T, R)
        if tr is not None:
            tr.mark("lm_head")
        return out

    def _lm_head(self, meta: StepMeta, ws: Workspace, T: int, R: int) -> torch.Tensor:
        rows = ws.final_bf16[:R]
        torch.index_select(ws.norm_out[:T], 0, meta.logits_idx[:R], out=rows)
        if isinstance(self.lm_head, L.MXWeight):
            L.quant_act(rows, out=ws.final_act.narrow(R))
            L.mx_linear(ws.final_act.narrow(R), self.lm_head, out=ws.logits_local[:R])
        else:
            L.bf16_linear(rows, self.lm_head, out=ws.logits_local[:R])
        return self.comm.all_gather_lastdim(ws.logits_local[:R], out=ws.logits[:R])
