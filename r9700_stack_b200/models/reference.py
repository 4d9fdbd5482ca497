"""Plain-PyTorch fp32 restatement of the hybrid decoder, used as the oracle for the fused kernels.

It reads the same weights as :class:`HybridLM` (dequantised to fp32) and applies the same
quantisation points (MXFP8 activations before MX GEMMs, e4m3 KV cache, bf16 residual stream), but
every op is a textbook torch expression: no custom kernel runs here.
"""
from __future__ import annotations

import torch
import torch.nn.functional as Fn

from ..ops import linear as L
from ..quant import formats as F


def fake_mxfp8(x: torch.Tensor) -> torch.Tensor:
    """Quantise rows to MXFP8 and back (block 32 along the last dim), in fp32 on x's device."""
    shp = x.shape
    b = x.float().reshape(-1, shp[-1] // 32, 32)
    amax = b.abs().amax(-1)
    e = F.mx_exponent(amax.cpu(), F.E4M3_MAX).to(x.device)
    s = torch.ldexp(torch.ones_like(amax), e)
    q = (b / s[..., None]).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    return (q * s[..., None]).reshape(shp)


def e4m3_roundtrip(x: torch.Tensor) -> torch.Tensor:
    return x.float().clamp(-448, 448).to(torch.float8_e4m3fn).float()


def bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def _w(w) -> torch.Tensor:
    if isinstance(w, (L.MXWeight, L.NVF4Weight)):
        return w.dequant()
    if isinstance(w, L.BF16Weight):
        return w.w.float()
    return w.float()


def _lin(x: torch.Tensor, w, mx: bool) -> torch.Tensor:
    xin = fake_mxfp8(x) if mx else bf16(x)
    return xin @ _w(w).T


def rmsnorm(x, w, eps, plus_one):
    wf = w.float() + (1.0 if plus_one else 0.0)
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * wf


class ReferenceState:
    def __init__(self, model):
        c = model.cfg
        self.k = {i: [] for i in c.attn_layers}
        self.v = {i: [] for i in c.attn_layers}
        self.ik = {i: [] for i in c.attn_layers}  # QSA indexer token keys (bf16 values)
        g = model.gdn_dims
        self.S = {i: torch.zeros(g["hv"], c.gdn_head_dim, c.gdn_head_dim, device=model.device) for i in c.gdn_layers}
        self.conv = {i: torch.zeros(g["conv_ch"], c.conv_width - 1, device=model.device) for i in c.gdn_layers}
        self.pos = 0


@torch.no_grad()
def reference_forward(model, tokens: list[int], st: ReferenceState, quantize_acts: bool = True) -> torch.Tensor:
    """Process `tokens` (continuing from `st`); returns fp32 logits [len(tokens), vocab_local].
    ``quantize_acts=False`` keeps the activations in full precision before MX GEMMs and the MX lm_head
    (the same weights, without the activation quantiser): the "truth" two differently-rounded runs of an
    MX model are both measured against."""
    c, dev = model.cfg, model.device
    mx = model.mx and quantize_acts
    T = len(tokens)
    pos = torch.arange(st.pos, st.pos + T, device=dev)
    resid = model.embed[torch.tensor(tokens, device=dev)].float()
    if c.hc_streams:
        return _forward_hc(model, tokens, st, pos, resid)
    y = None
    for i, lay in enumerate(model.layers):
        if y is not None:
            resid = bf16(resid + y)
        h = rmsnorm(resid, lay["in_norm"], c.rms_eps, c.norm_plus_one)
        y = _mixer(model, i, lay, h, pos, st, mx)
        resid = bf16(resid + y)
        h = rmsnorm(resid, lay["post_norm"], c.rms_eps, c.norm_plus_one)
        y = _ffn(model, i, lay, h, tokens, mx)
    resid = bf16(resid + y)
    h = bf16(rmsnorm(resid, model.final_norm, c.rms_eps, c.norm_plus_one))
    return _finish(model, h, st, T, quantize_acts)


def _mixer(model, i, lay, h, pos, st, mx):
    if lay["attn"]:
        return bf16(_attn(model, i, lay, h, pos, st, mx))
    return bf16(_gdn(model, i, lay, h, st, mx))


def _ffn(model, i, lay, h, tokens, mx):
    c, dev = model.cfg, model.device
    if "router" in lay:
        y = _moe(model, lay, bf16(h))
        if getattr(model, "ple", None) is not None:
            y = bf16(y)
            ids = torch.tensor(tokens, device=dev) * c.layers + i
            p = model.ple.gather_ref(ids).to(dev)
            g = bf16(bf16(h) @ lay["ple_gate"].w.float().T)
            hh = bf16(torch.nn.functional.gelu(g, approximate="tanh") * bf16(p))
            y = y + hh @ lay["ple_out"].w.float().T
        return bf16(y)
    g = _lin(h, lay["w_gate"], mx)
    u = _lin(h, lay["w_up"], mx)
    return bf16(_lin(Fn.silu(g) * u, lay["w_down"], mx))


def _finish(model, h, st, T, quantize_acts: bool = True):
    c = model.cfg
    lm_mx = isinstance(model.lm_head, L.MXWeight) and quantize_acts
    logits = (fake_mxfp8(h) if lm_mx else h) @ _w(model.lm_head).T
    st.pos += T
    # recurrent state is stored in the state dtype between steps
    if c.gdn_state_dtype == "bf16":
        for k in st.S:
            st.S[k] = bf16(st.S[k])
            st.conv[k] = bf16(st.conv[k])
    return logits


def _hc_point(model, p, X, y):
    """Hyper-connection norm point: (new residual streams, next block input), both bf16 values."""
    from ..ops import hc as HCo

    c = model.cfg
    l = bf16(y) @ p.wl.w.float().T if y is not None else None
    X, N = HCo.combine_norm_ref(X, y, l, p.w, c.hc_streams, c.rms_eps)
    return X, HCo.gate_mix_ref(N, p.g, c.hc_streams).float()


def _forward_hc(model, tokens, st, pos, emb):
    c, mx = model.cfg, model.mx
    T, HC = len(tokens), c.hc_streams
    X = emb.bfloat16().repeat(1, HC)
    y = None
    for i, lay in enumerate(model.layers):
        X, h = _hc_point(model, lay["hc_in"], X, y)
        y = _mixer(model, i, lay, h, pos, st, mx)
        X, h = _hc_point(model, lay["hc_post"], X, y)
        y = _ffn(model, i, lay, h, tokens, mx)
    X, h = _hc_point(model, model.hc_final, X, y)
    return _finish(model, h, st, T)


def _rope(x, pos, rot, theta):
    half = rot // 2
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float64, device=x.device) / rot))
    f = torch.outer(pos.double(), inv).float()
    cos, sin = f.cos()[:, None, :], f.sin()[:, None, :]
    x1, x2 = x[..., :half], x[..., half:rot]
    out = x.clone()
    out[..., :half] = x1 * cos - x2 * sin
    out[..., half:rot] = x2 * cos + x1 * sin
    return out


def _attn(model, i, lay, h, pos, st, mx):
    c, a = model.cfg, model.attn_dims
    hq, hkv, D = a["hq"], a["hkv"], c.head_dim
    T = h.shape[0]
    qkv = bf16(_lin(h, lay["w_qkv"], mx))
    q = qkv[:, : hq * D].reshape(T, hq, D)
    gate = qkv[:, hq * D : 2 * hq * D]
    k_off = 2 * hq * D
    k = qkv[:, k_off : k_off + hkv * D].reshape(T, hkv, D)
    v = qkv[:, k_off + hkv * D : k_off + 2 * hkv * D].reshape(T, hkv, D)
    q = bf16(rmsnorm(q, lay["q_norm"], c.rms_eps, c.norm_plus_one))
    k = bf16(rmsnorm(k, lay["k_norm"], c.rms_eps, c.norm_plus_one))
    q = bf16(_rope(q, pos, c.rotary_dim, c.rope_theta))
    k = _rope(k, pos, c.rotary_dim, c.rope_theta)
    st.k[i].append(e4m3_roundtrip(bf16(k)))
    st.v[i].append(e4m3_roundtrip(v))
    K = torch.cat(st.k[i], 0)  # [ctx, hkv, D]
    V = torch.cat(st.v[i], 0)
    ctx = K.shape[0]
    G = hq // hkv
    Kx = K.repeat_interleave(G, dim=1)
    Vx = V.repeat_interleave(G, dim=1)
    s = torch.einsum("thd,chd->thc", q, Kx) * model.sm_scale
    qpos = pos[:, None]
    kpos = torch.arange(ctx, device=h.device)[None, :]
    allowed = kpos <= qpos
    if c.qsa_topk:
        allowed = allowed & _qsa_mask(model, i, lay, h, pos, st, mx, ctx)
    s = s.masked_fill((~allowed)[:, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("thc,chd->thd", p, Vx).reshape(T, hq * D)
    o = bf16(o * torch.sigmoid(gate))
    return _lin(o, lay["w_o"], mx)


def _qsa_mask(model, i, lay, h, pos, st, mx, ctx):
    """QSA key mask [T, ctx]: the top-k complete 4-token groups by the indexer score plus the open
    group's causal tail, for every query row."""
    c = model.cfg
    Hi, k = c.qsa_heads, c.qsa_topk
    T = h.shape[0]
    pj = bf16(_lin(h, lay["w_idx"], mx)).reshape(T, Hi + 1, 128)
    pj = bf16(rmsnorm(pj, lay["idx_norm"], c.rms_eps, c.norm_plus_one))
    pj = bf16(_rope(pj, pos, 64, c.rope_theta))
    iq, ik = pj[:, :Hi], pj[:, Hi]
    st.ik[i].append(ik)
    IK = torch.cat(st.ik[i], 0)  # [ctx, 128]
    ng = ctx // 4
    ck = e4m3_roundtrip(IK[: 4 * ng].reshape(ng, 4, 128).sum(1) * 0.25) if ng else IK[:0]
    mask = torch.zeros(T, ctx, dtype=torch.bool, device=h.device)
    for t in range(T):
        p = int(pos[t])
        vis = (p + 1) // 4
        if vis > k:
            sc = (torch.relu(iq[t] @ ck[:vis].T) * 128 ** -0.5).sum(0)
            sel = torch.topk(sc, k).indices
        else:
            sel = torch.arange(vis, device=h.device)
        g = torch.zeros(ctx, dtype=torch.bool, device=h.device)
        idx = (sel[:, None] * 4 + torch.arange(4, device=h.device)[None, :]).reshape(-1)
        g[idx] = True
        g[4 * vis : p + 1] = True
        mask[t] = g
    return mask


def _gdn(model, i, lay, h, st, mx):
    c, g = model.cfg, model.gdn_dims
    hk, hv, d = g["hk"], g["hv"], c.gdn_head_dim
    T = h.shape[0]
    proj = bf16(_lin(h, lay["w_in"], mx))
    C = g["conv_ch"]
    x = proj[:, :C]
    z_off = 2 * hk * d + hv * d
    z = proj[:, z_off : z_off + hv * d].reshape(T, hv, d)
    b = proj[:, z_off + hv * d : z_off + hv * d + hv]
    a = proj[:, z_off + hv * d + hv : z_off + hv * d + 2 * hv]
    W = c.conv_width
    full = torch.cat([st.conv[i].T, x], 0)  # [(W-1) + T, C]
    cw = lay["conv_w"].float()
    conv = torch.stack([(full[t : t + W] * cw.T).sum(0) for t in range(T)], 0)
    st.conv[i] = full[-(W - 1) :].T.clone()
    conv = Fn.silu(conv)
    q = conv[:, : hk * d].reshape(T, hk, d)
    k = conv[:, hk * d : 2 * hk * d].reshape(T, hk, d)
    v = conv[:, 2 * hk * d :].reshape(T, hv, d)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * (d**-0.5)
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    gg = -torch.exp(lay["A_log"]) * Fn.softplus(a + lay["dt_bias"])
    beta = torch.sigmoid(b)
    rep = hv // hk
    S = st.S[i]
    outs = []
    for t in range(T):
        kt = k[t].repeat_interleave(rep, 0)  # [hv, d]
        qt = q[t].repeat_interleave(rep, 0)
        S = S * torch.exp(gg[t])[:, None, None]
        kv = torch.einsum("hij,hi->hj", S, kt)
        delta = beta[t][:, None] * (v[t] - kv)
        S = S + kt[:, :, None] * delta[:, None, :]
        outs.append(torch.einsum("hij,hi->hj", S, qt))
    st.S[i] = S
    o = torch.stack(outs, 0)  # [T, hv, d]
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + c.rms_eps) * lay["gdn_norm"].float() * Fn.silu(z)
    o = bf16(o.reshape(T, hv * d))
    return _lin(o, lay["w_out"], mx)


def _moe(model, lay, x):
    """Routed experts (softmax top-k, renormalised) + sigmoid-gated shared expert, fp32 math."""
    c = model.cfg
    T = x.shape[0]
    logits = bf16(x) @ lay["router"].w.float().T
    p = torch.softmax(logits, -1)
    w, ids = torch.topk(p, c.moe_topk, dim=-1)
    w = w / w.sum(-1, keepdim=True)
    xq = fake_mxfp8(x)
    I, El = c.moe_ffn, model.e_local
    G = lay["e_gate"].dequant().view(El, I, -1)
    U = lay["e_up"].dequant().view(El, I, -1)
    D = lay["e_down"].dequant().view(El, c.hidden, I)
    out = torch.zeros(T, c.hidden, device=x.device)
    for t in range(T):
        for j in range(c.moe_topk):
            e = model.local_index(int(ids[t, j]))
            if e < 0:
                continue
            hh = Fn.silu(xq[t] @ G[e].T) * (xq[t] @ U[e].T)
            out[t] += w[t, j] * (fake_mxfp8(hh[None])[0] @ D[e].T).to(torch.bfloat16).float()
    if "s_gate" in lay:
        sh = bf16(Fn.silu(x @ lay["s_gate"].w.float().T) * (x @ lay["s_up"].w.float().T))
        sh = bf16(sh @ lay["s_down"].w.float().T)
        gt = torch.sigmoid(x @ lay["s_gvec"].w.float().T)
        out = out + gt * sh
    return out
