"""Plain-PyTorch fp32 restatement of the sparse-MLA MoE decoder (oracle for ``MLAMoELM``).

Same weights, same storage roundings (bf16 activations between ops, bf16 latent rows, e4m3
indexer keys, MXFP8 activations into the MX experts); attention is computed densely over the top-k
positions that the indexer selects.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as Fn

from .reference import bf16, fake_mxfp8

LAT, PE = 512, 64


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _rope(x, pos, cs):
    c, s = cs[pos, :32], cs[pos, 32:]
    while c.dim() < x.dim():
        c, s = c.unsqueeze(-2), s.unsqueeze(-2)
    a, b = x[..., :32], x[..., 32:64]
    return torch.cat([a * c - b * s, b * c + a * s, x[..., 64:]], -1)


class MLARefState:
    def __init__(self, model):
        self.lat = {i: [] for i in range(model.cfg.layers)}
        self.ik = {i: [] for i in range(model.cfg.layers)}
        self.pos = 0


def _route(x, lay, c, mode: int = 1):
    """Group-limited top-k over biased scores; mode 1: sigmoid scores (GLM / DeepSeek-V3 class),
    mode 2: sqrt(softplus) scores (DeepSeek-V4 class)."""
    logits = bf16(x) @ lay["router"].w.float().T
    s = torch.sigmoid(logits) if mode == 1 else torch.sqrt(Fn.softplus(logits))
    b = s + lay["router_bias"].float()
    T, E = b.shape
    g = b.view(T, c.n_group, -1).topk(2, -1).values.sum(-1)
    keep = torch.zeros(T, c.n_group, dtype=torch.bool, device=x.device)
    keep.scatter_(1, g.topk(c.topk_group, -1).indices, True)
    b = b.masked_fill(~keep.repeat_interleave(E // c.n_group, 1), float("-inf"))
    ids = b.topk(c.moe_topk, -1).indices
    w = s.gather(1, ids)
    return ids, w / w.sum(-1, keepdim=True) * c.routed_scale


def _attention_ref(model, lay, i: int, h: torch.Tensor, pos: torch.Tensor, st: MLARefState) -> torch.Tensor:
    """One sparse-MLA attention sublayer (indexer, top-k, softmax over the selected latent rows,
    W_uv and the output projection) on normalised bf16 input h [T, H]; returns y (bf16 values)."""
    c = model.cfg
    T = h.shape[0]
    cs = model.cos_sin
    cq = bf16(_rms(bf16(h @ lay["w_dq"].w.float().T), lay["q_norm"], c.rms_eps))
    q = bf16(cq @ lay["w_uq"].w.float().T).view(T, model.nh, c.qk_nope + PE)
    qpe = bf16(_rope(q[..., c.qk_nope:], pos, cs))
    qlat = bf16(torch.einsum("thk,hnk->thn", q[..., : c.qk_nope], lay["w_uk"].float()))
    kv = bf16(h @ lay["w_dkv"].w.float().T)
    lat = torch.cat([bf16(_rms(kv[:, :LAT], lay["kv_norm"], c.rms_eps)), bf16(_rope(kv[:, LAT:], pos, cs))], -1)
    ik = bf16(h @ lay["w_ik"].w.float().T)
    ik = _rope(_rms(ik, lay["ik_norm"], c.rms_eps), pos, cs).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    st.lat[i].append(lat)
    st.ik[i].append(ik)
    LAT_all, IK_all = torch.cat(st.lat[i]), torch.cat(st.ik[i])
    qi = bf16(cq @ lay["w_iq"].w.float().T).view(T, c.index_heads, 128)
    qi = bf16(_rope(qi, pos, cs))
    wi = (h @ lay["w_iw"].w.float().T) / math.sqrt(c.index_heads * 128)
    outs = []
    for t in range(T):
        ctx = int(pos[t]) + 1
        sc = (wi[t][:, None] * torch.relu(qi[t] @ IK_all[:ctx].T)).sum(0)
        sel = torch.topk(sc, min(c.index_topk, ctx)).indices
        R = LAT_all[sel]
        qf = torch.cat([qlat[t], qpe[t]], -1)
        p = torch.softmax((qf @ R.T) * model.scale, -1)
        outs.append(bf16(p @ R[:, :LAT]))
    olat = torch.stack(outs)
    o = bf16(torch.einsum("thk,hnk->thn", olat, lay["w_uv"].float())).reshape(T, -1)
    return bf16(o @ lay["w_o"].w.float().T)


@torch.no_grad()
def reference_forward_mla(model, tokens: list[int], st: MLARefState) -> torch.Tensor:
    c, dev = model.cfg, model.device
    T = len(tokens)
    pos = torch.arange(st.pos, st.pos + T, device=dev)
    resid = model.embed[torch.tensor(tokens, device=dev)].float()
    y = None
    for i, lay in enumerate(model.layers):
        if y is not None:
            resid = bf16(resid + y)
        h = bf16(_rms(resid, lay["in_norm"], c.rms_eps))
        y = _attention_ref(model, lay, i, h, pos, st)
        resid = bf16(resid + y)
        h = bf16(_rms(resid, lay["post_norm"], c.rms_eps))
        if "w_gate" in lay:
            a = bf16(Fn.silu(h @ lay["w_gate"].w.float().T) * (h @ lay["w_up"].w.float().T))
            y = bf16(a @ lay["w_down"].w.float().T)
        else:
            ids, w = _route(h, lay, c)
            I, El = c.moe_ffn, model.e_local
            G = lay["e_gate"].dequant().view(El, I, -1)
            U = lay["e_up"].dequant().view(El, I, -1)
            D = lay["e_down"].dequant().view(El, c.hidden, I)
            xq = fake_mxfp8(h)
            out = torch.zeros(T, c.hidden, device=dev)
            for t in range(T):
                for j in range(c.moe_topk):
                    e = int(ids[t, j])
                    hh = Fn.silu(xq[t] @ G[e].T) * (xq[t] @ U[e].T)
                    out[t] += w[t, j] * bf16(fake_mxfp8(hh[None])[0] @ D[e].T)
            sh = bf16(Fn.silu(h @ lay["s_gate"].w.float().T) * (h @ lay["s_up"].w.float().T))
            out = out + bf16(sh @ lay["s_down"].w.float().T)
            y = bf16(out)
    resid = bf16(resid + y)
    hf = bf16(_rms(resid, model.final_norm, c.rms_eps))
    st.pos += T
    return hf @ model.lm_head.w.float().T


class DSV4RefState(MLARefState):
    def __init__(self, model):
        super().__init__(model)
        self.tokens: list[int] = []


def _ngram_ref(history: list[int], order: int, rows: int) -> int:
    """Hash of the last ``order`` tokens of a sequence (missing history counts as -1), the device
    kernel's multiplicative hash written out."""
    win = ([-1] * order + history)[-order:]
    h = order
    for v in win:
        h = (h * 1000003 + v + 1) & 0x7FFFFFFFFFFF
    return h % rows


def _engram_ref(model, lay, h: torch.Tensor, st: DSV4RefState, T: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(gate logits [T, 1] fp32, projected n-gram embedding [T, H] bf16 values) for the step's tokens."""
    c = model.cfg
    toks = st.tokens
    base = len(toks) - T
    ids = [[_ngram_ref(toks[: base + t + 1], o + 2, c.engram_rows) for o in range(c.engram_orders)] for t in range(T)]
    rows = bf16(lay["engram"].gather_ref(torch.tensor(ids).view(-1)).to(h.device)).view(T, c.engram_orders, -1)
    esum = bf16(rows.sum(1))
    gate = h @ lay["eng_gate"].w.float().T
    return gate, bf16(esum @ lay["eng_proj"].w.float().T)


def _trellis_moe_ref(model, lay, h: torch.Tensor) -> torch.Tensor:
    """Routed experts in trellis codes (dense fp32 dequant of every used expert) + the shared expert."""
    from ..quant import exl3 as E

    c, dev = model.cfg, model.device
    T = h.shape[0]
    ids, w = _route(h, lay, c, mode=2)
    e0 = model.par.tp_rank * model.e_local
    cache = {}

    def dense(name, e):
        key = (name, e)
        if key not in cache:
            x = lay[name]
            cache[key] = E.dequant(x.trellis[e].cpu(), x.suh[e].cpu(), x.svh[e].cpu(), x.K, x.cb).to(dev)  # [in, out]
        return cache[key]

    out = torch.zeros(T, c.hidden, device=dev)
    for t in range(T):
        for j in range(c.moe_topk):
            e = int(ids[t, j]) - e0
            if not 0 <= e < model.e_local:
                continue
            hh = bf16(Fn.silu(h[t] @ dense("x_gate", e)) * (h[t] @ dense("x_up", e)))
            out[t] += w[t, j] * bf16(hh @ dense("x_down", e))
    sh = bf16(Fn.silu(h @ lay["s_gate"].w.float().T) * (h @ lay["s_up"].w.float().T))
    return bf16(out + bf16(sh @ lay["s_down"].w.float().T))


@torch.no_grad()
def reference_forward_dsv4(model, tokens: list[int], st: DSV4RefState) -> torch.Tensor:
    """fp32 restatement of ``DSV4LM`` (one sequence): mHC seams over the residual streams
    (``ops.mhc.seam_ref``), sparse-MLA attention, Engram n-gram embeddings at the Engram layers,
    trellis-coded routed experts dequantised densely, the head seam and the final norm."""
    from ..ops.mhc import seam_ref

    c, dev = model.cfg, model.device
    T = len(tokens)
    st.tokens += list(tokens)
    pos = torch.arange(st.pos, st.pos + T, device=dev)
    e = model.embed[torch.tensor(tokens, device=dev)]
    R = e[:, None, :].expand(T, c.hc, c.hidden).contiguous()
    so = post = comb = None
    for i, lay in enumerate(model.layers):
        R, pa, ca, li = seam_ref(R, lay["hc_attn"], so, post, comb)
        h = bf16(_rms(li.float(), lay["in_norm"], c.rms_eps))
        y = _attention_ref(model, lay, i, h, pos, st)
        if "engram" in lay:
            gate, y2 = _engram_ref(model, lay, h, st, T)
            y = bf16(y + y2 * torch.sigmoid(gate))
        R, pf, cf, li = seam_ref(R, lay["hc_ffn"], y.to(torch.bfloat16), pa, ca)
        h = bf16(_rms(li.float(), lay["post_norm"], c.rms_eps))
        if "router" in lay:
            y = _trellis_moe_ref(model, lay, h)
        else:
            a = bf16(Fn.silu(h @ lay["w_gate"].w.float().T) * (h @ lay["w_up"].w.float().T))
            y = bf16(a @ lay["w_down"].w.float().T)
        so, post, comb = y.to(torch.bfloat16), pf, cf
    _, _, _, li = seam_ref(R, model.hc_head, so, post, comb)
    hf = bf16(_rms(li.float(), model.final_norm, c.rms_eps))
    st.pos += T
    return hf @ model.lm_head.w.float().T
