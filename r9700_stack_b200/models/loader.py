"""Checkpoint loading: Hugging Face safetensors shards -> this framework's device formats.

Names follow the Hugging Face Qwen3-Next hybrid layout (``model.layers.{i}.linear_attn.*`` for Gated
DeltaNet layers, ``model.layers.{i}.self_attn.*`` for gated attention, ``mlp.*`` dense or
``mlp.experts.{e}.*`` / ``mlp.shared_expert.*`` MoE). A quantised linear appears as
  * compressed-tensors NVFP4: ``weight_packed`` u8 [N, K/2] (e2m1 pairs), ``weight_scale`` e4m3 [N, K/16],
    ``weight_global_scale`` f32 (w = v * s / g)  -> MXFP4 at load (the reference's conversion);
  * block fp8: ``weight`` e4m3 [N, K] + ``weight_scale_inv`` f32 [N/128, K/128]   -> MXFP8 at load;
  * plain ``weight`` (bf16 / fp16 / fp32)                                       -> the model's format.
Tensor-parallel ranks take their slices while loading (head-grouped rows for the merged GDN and
attention projections, columns for the row-parallel outputs, expert ranges for MoE).
``dry_run(path, cfg)`` maps every tensor name without reading data and reports unmapped or missing
names; ``export_hf(model, path)`` writes a model in the same layout (bf16), which is what the
round-trip tests load. The HF layout is reproduced from its public model definition; the in_proj
packing ([q_g, k_g, v_g, z_g] per key head g, then [b_g, a_g]) and the attention q/gate interleave
are the parts that must match a published checkpoint.
Reference: r9700_vllm/quant/ct.py:347-462, quant/nvfp4.py:78-112, linear/fp8_block.py:23,
models/deepseek_v41_exl3.py:194-417 (loader with a name-mapping dry run).
"""
from __future__ import annotations

import glob
import json
import os
import re
from dataclasses import dataclass

import torch

from ..ops import linear as L

_LAYER = re.compile(r"^model\.layers\.(\d+)\.(.+)$")


@dataclass
class Entry:
    name: str
    shard: str
    shape: tuple
    dtype: str


def index(path: str) -> dict[str, Entry]:
    """name -> Entry over every *.safetensors file of a checkpoint directory (headers only)."""
    from safetensors import safe_open

    out = {}
    for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
        with safe_open(f, framework="pt") as sf:
            for k in sf.keys():
                sl = sf.get_slice(k)
                out[k] = Entry(k, f, tuple(sl.get_shape()), str(sl.get_dtype()))
    return out


def _linear_stem(name: str) -> tuple[str, str] | None:
    for suf in ("weight_packed", "weight_scale", "weight_global_scale", "weight_scale_inv", "weight"):
        if name.endswith("." + suf):
            return name[: -len(suf) - 1], suf
    return None


# ------------------------------------------------------------------------------------------------
# mapping: HF module stems of one layer -> (our key, role)
# ------------------------------------------------------------------------------------------------
def layer_targets(cfg, i: int) -> dict[str, str]:
    """HF stem (below model.layers.{i}.) -> our layer key."""
    t = {"input_layernorm": "in_norm", "post_attention_layernorm": "post_norm"}
    if cfg.is_attention(i):
        t.update({"self_attn.q_proj": "w_qkv:q", "self_attn.k_proj": "w_qkv:k", "self_attn.v_proj": "w_qkv:v",
                  "self_attn.o_proj": "w_o", "self_attn.q_norm": "q_norm", "self_attn.k_norm": "k_norm"})
    else:
        t.update({"linear_attn.in_proj_qkvz": "w_in:qkvz", "linear_attn.in_proj_ba": "w_in:ba",
                  "linear_attn.conv1d": "conv_w", "linear_attn.A_log": "A_log", "linear_attn.dt_bias": "dt_bias",
                  "linear_attn.norm": "gdn_norm", "linear_attn.out_proj": "w_out"})
    if cfg.moe_experts:
        t.update({"mlp.gate": "router", "mlp.shared_expert.gate_proj": "s_gate", "mlp.shared_expert.up_proj": "s_up",
                  "mlp.shared_expert.down_proj": "s_down", "mlp.shared_expert_gate": "s_gvec"})
        for e in range(cfg.moe_experts):
            for p, k in (("gate_proj", "e_gate"), ("up_proj", "e_up"), ("down_proj", "e_down")):
                t[f"mlp.experts.{e}.{p}"] = f"{k}:{e}"
    else:
        t.update({"mlp.gate_proj": "w_gate", "mlp.up_proj": "w_up", "mlp.down_proj": "w_down"})
    return t


def dry_run(path: str, cfg) -> dict:
    """Map every checkpoint tensor to a model slot without reading data."""
    idx = index(path)
    mapped, unmapped = {}, []
    expected = {"model.embed_tokens", "model.norm", "lm_head"}
    for i in range(cfg.layers):
        expected |= {f"model.layers.{i}.{s}" for s in layer_targets(cfg, i)}
    seen = set()
    for name in idx:
        st = _linear_stem(name)
        stem = st[0] if st else name
        if stem in ("model.embed_tokens", "model.norm", "lm_head") or (
                (m := _LAYER.match(stem)) and m.group(2) in layer_targets(cfg, int(m.group(1)))):
            mapped[name] = stem
            seen.add(stem)
        elif stem.endswith(("A_log", "dt_bias")) and _LAYER.match(stem):
            mapped[name] = stem
            seen.add(stem)
        else:
            unmapped.append(name)
    missing = sorted(expected - seen)
    return {"tensors": len(idx), "mapped": len(mapped), "unmapped": unmapped, "missing": missing}


# ------------------------------------------------------------------------------------------------
# reading and converting
# ------------------------------------------------------------------------------------------------
class _Reader:
    def __init__(self, path: str):
        from safetensors import safe_open

        self.idx = index(path)
        self._open = {}
        self._safe_open = safe_open

    def has(self, name: str) -> bool:
        return name in self.idx

    def get(self, name: str) -> torch.Tensor:
        e = self.idx[name]
        if e.shard not in self._open:
            self._open[e.shard] = self._safe_open(e.shard, framework="pt")
        return self._open[e.shard].get_tensor(name)


def _float_weight(rd: _Reader, stem: str, device) -> torch.Tensor:
    """A linear's weight as fp32 [N, K] on the device, whatever its checkpoint format."""
    from ..quant import formats as F

    if rd.has(stem + ".weight_packed"):
        packed = rd.get(stem + ".weight_packed").to(device)
        s16 = rd.get(stem + ".weight_scale").view(torch.uint8).to(device)
        g = float(rd.get(stem + ".weight_global_scale").float().reshape(-1)[0])
        return F.dequant_nvfp4(packed, s16, g).to(device)
    w = rd.get(stem + ".weight")
    if rd.has(stem + ".weight_scale_inv"):
        s = rd.get(stem + ".weight_scale_inv").float()
        q = w.float()
        srep = s.repeat_interleave(128, 0)[: q.shape[0]].repeat_interleave(128, 1)[:, : q.shape[1]]
        return (q * srep).to(device)
    return w.float().to(device)


def _convert(rd: _Reader, stem: str, fmt: str, rows: slice | list | None, cols: slice | None, device):
    """Load a linear (optionally a TP slice) into the model's device format."""
    from .weights import from_float

    if fmt != "bf16" and rd.has(stem + ".weight_packed") and rows is None and cols is None:
        # NVFP4 straight to MXFP4 (the load-time conversion of the published checkpoints)
        packed = rd.get(stem + ".weight_packed").to(device)
        s16 = rd.get(stem + ".weight_scale").view(torch.uint8).to(device)
        g = float(rd.get(stem + ".weight_global_scale").float().reshape(-1)[0])
        mw = L.mx_from_nvfp4(packed, s16, g, search=True)
        return mw.to_tiled()
    w = _float_weight(rd, stem, device)
    if rows is not None:
        w = w[rows]
    if cols is not None:
        w = w[:, cols]
    return from_float(w.contiguous(), "bf16" if fmt == "bf16" else ("nvfp4" if fmt == "nvfp4" else fmt))


def load_into(model, path: str) -> dict:
    """Overwrite a constructed HybridLM / HybridMoELM's weights with a checkpoint's. Returns stats."""
    cfg, par, dev = model.cfg, model.par, model.device
    rd = _Reader(path)
    tp, r = par.tp_size, par.tp_rank
    fmt = cfg.weight_format
    n = 0
    model.embed = rd.get("model.embed_tokens.weight").to(dev, torch.bfloat16)
    model.final_norm = rd.get("model.norm.weight").to(dev, torch.bfloat16)
    V = model.vocab_local
    model.lm_head = _convert(rd, "lm_head", cfg.lm_head_format if cfg.lm_head_format != "block_fp8" else "mxfp8",
                             slice(r * V, (r + 1) * V) if tp > 1 else None, None, dev)
    for i, lay in enumerate(model.layers):
        p = f"model.layers.{i}."
        lay["in_norm"] = rd.get(p + "input_layernorm.weight").to(dev, torch.bfloat16)
        lay["post_norm"] = rd.get(p + "post_attention_layernorm.weight").to(dev, torch.bfloat16)
        if lay["attn"]:
            a, D = model.attn_dims, cfg.head_dim
            hq, hkv = a["hq"], a["hkv"]
            q = _float_weight(rd, p + "self_attn.q_proj", dev).view(cfg.n_q_heads, 2 * D, -1)
            q = q[r * hq:(r + 1) * hq]
            k = _float_weight(rd, p + "self_attn.k_proj", dev).view(cfg.n_kv_heads, D, -1)
            v = _float_weight(rd, p + "self_attn.v_proj", dev).view(cfg.n_kv_heads, D, -1)
            kv0 = (r * hkv) % cfg.n_kv_heads if tp > cfg.n_kv_heads else r * hkv
            k, v = k[kv0:kv0 + hkv], v[kv0:kv0 + hkv]
            w = torch.cat([q[:, :D].reshape(-1, q.shape[-1]), q[:, D:].reshape(-1, q.shape[-1]),
                           k.reshape(-1, k.shape[-1]), v.reshape(-1, v.shape[-1])], 0)
            from .weights import from_float

            lay["w_qkv"] = from_float(w.contiguous(), fmt)
            Ko = hq * D
            lay["w_o"] = _convert(rd, p + "self_attn.o_proj", fmt, None, slice(r * Ko, (r + 1) * Ko), dev)
            lay["q_norm"] = rd.get(p + "self_attn.q_norm.weight").to(dev, torch.bfloat16)
            lay["k_norm"] = rd.get(p + "self_attn.k_norm.weight").to(dev, torch.bfloat16)
        else:
            g, d = model.gdn_dims, cfg.gdn_head_dim
            HK, HV = cfg.gdn_k_heads, cfg.gdn_v_heads
            rep = HV // HK
            hk = g["hk"]
            qkvz = _float_weight(rd, p + "linear_attn.in_proj_qkvz", dev).view(HK, 2 * d + 2 * rep * d, -1)
            ba = _float_weight(rd, p + "linear_attn.in_proj_ba", dev).view(HK, 2 * rep, -1)
            qkvz, ba = qkvz[r * hk:(r + 1) * hk], ba[r * hk:(r + 1) * hk]
            qw, kw = qkvz[:, :d], qkvz[:, d:2 * d]
            vw, zw = qkvz[:, 2 * d:2 * d + rep * d], qkvz[:, 2 * d + rep * d:]
            bw, aw = ba[:, :rep], ba[:, rep:]
            Kd = qkvz.shape[-1]
            w = torch.cat([qw.reshape(-1, Kd), kw.reshape(-1, Kd), vw.reshape(-1, Kd), zw.reshape(-1, Kd),
                           bw.reshape(-1, Kd), aw.reshape(-1, Kd)], 0)
            from .weights import from_float

            lay["w_in"] = from_float(w.contiguous(), fmt)
            conv = rd.get(p + "linear_attn.conv1d.weight").float().reshape(-1, cfg.conv_width)
            C = HK * d
            qc, kc, vc = conv[:C], conv[C:2 * C], conv[2 * C:]
            vd = HV // tp * d
            lay["conv_w"] = torch.cat([qc[r * hk * d:(r + 1) * hk * d], kc[r * hk * d:(r + 1) * hk * d],
                                       vc[r * vd:(r + 1) * vd]], 0).to(dev, torch.bfloat16).contiguous()
            hv = g["hv"]
            lay["A_log"] = rd.get(p + "linear_attn.A_log").float().to(dev)[r * hv:(r + 1) * hv].contiguous()
            lay["dt_bias"] = rd.get(p + "linear_attn.dt_bias").float().to(dev)[r * hv:(r + 1) * hv].contiguous()
            lay["gdn_norm"] = rd.get(p + "linear_attn.norm.weight").to(dev, torch.bfloat16)
            Ko = hv * d
            lay["w_out"] = _convert(rd, p + "linear_attn.out_proj", fmt, None, slice(r * Ko, (r + 1) * Ko), dev)
        if not cfg.moe_experts:
            F_ = model.ffn_local
            rows = slice(r * F_, (r + 1) * F_) if tp > 1 else None
            lay["w_gate"] = _convert(rd, p + "mlp.gate_proj", fmt, rows, None, dev)
            lay["w_up"] = _convert(rd, p + "mlp.up_proj", fmt, rows, None, dev)
            lay["w_down"] = _convert(rd, p + "mlp.down_proj", fmt, None, slice(r * F_, (r + 1) * F_) if tp > 1 else None, dev)
        else:
            from .weights import from_float

            El, e0 = model.e_local, r * model.e_local
            lay["router"] = L.BF16Weight(rd.get(p + "mlp.gate.weight").to(dev, torch.bfloat16))
            for key, hf in (("e_gate", "gate_proj"), ("e_up", "up_proj"), ("e_down", "down_proj")):
                ws = [_float_weight(rd, p + f"mlp.experts.{e}.{hf}", dev) for e in range(e0, e0 + El)]
                lay[key] = from_float(torch.cat(ws, 0).contiguous(), "nvfp4", tiled=True)
            if model.shared_local:
                S_ = model.shared_local
                sl = slice(r * S_, (r + 1) * S_)
                lay["s_gate"] = L.BF16Weight(_float_weight(rd, p + "mlp.shared_expert.gate_proj", dev)[sl].to(torch.bfloat16).contiguous())
                lay["s_up"] = L.BF16Weight(_float_weight(rd, p + "mlp.shared_expert.up_proj", dev)[sl].to(torch.bfloat16).contiguous())
                lay["s_down"] = L.BF16Weight(_float_weight(rd, p + "mlp.shared_expert.down_proj", dev)[:, sl].to(torch.bfloat16).contiguous())
                lay["s_gvec"] = L.BF16Weight(rd.get(p + "mlp.shared_expert_gate.weight").to(dev, torch.bfloat16))
        n += 1
    return {"layers": n}


# ------------------------------------------------------------------------------------------------
# export (bf16): the inverse mapping, for round-trip tests and for handing a synthetic model on
# ------------------------------------------------------------------------------------------------
def _dense(w) -> torch.Tensor:
    if isinstance(w, L.MXWeight):
        return w.dequant()
    if isinstance(w, L.BF16Weight):
        return w.w.float()
    return w.float()


def export_hf(model, path: str) -> None:
    """Write a single-rank model in the HF hybrid layout (bf16 safetensors + config.json)."""
    from safetensors.torch import save_file

    assert model.par.tp_size == 1
    cfg = model.cfg
    os.makedirs(path, exist_ok=True)
    t = {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.final_norm,
         "lm_head.weight": _dense(model.lm_head).bfloat16()}
    for i, lay in enumerate(model.layers):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = lay["in_norm"]
        t[p + "post_attention_layernorm.weight"] = lay["post_norm"]
        if lay["attn"]:
            a, D = model.attn_dims, cfg.head_dim
            hq, hkv = a["hq"], a["hkv"]
            w = _dense(lay["w_qkv"])
            q, gt = w[: hq * D].view(hq, D, -1), w[hq * D: 2 * hq * D].view(hq, D, -1)
            t[p + "self_attn.q_proj.weight"] = torch.cat([q, gt], 1).reshape(-1, w.shape[1]).bfloat16()
            t[p + "self_attn.k_proj.weight"] = w[2 * hq * D: 2 * hq * D + hkv * D].bfloat16()
            t[p + "self_attn.v_proj.weight"] = w[2 * hq * D + hkv * D:].bfloat16()
            t[p + "self_attn.o_proj.weight"] = _dense(lay["w_o"]).bfloat16()
            t[p + "self_attn.q_norm.weight"] = lay["q_norm"]
            t[p + "self_attn.k_norm.weight"] = lay["k_norm"]
        else:
            g, d = model.gdn_dims, cfg.gdn_head_dim
            hk, hv = g["hk"], g["hv"]
            rep = hv // hk
            w = _dense(lay["w_in"])
            K = w.shape[1]
            C = hk * d
            qw, kw = w[:C].view(hk, d, K), w[C:2 * C].view(hk, d, K)
            vw = w[2 * C:2 * C + hv * d].view(hk, rep * d, K)
            zw = w[2 * C + hv * d:2 * C + 2 * hv * d].view(hk, rep * d, K)
            bw = w[2 * C + 2 * hv * d:2 * C + 2 * hv * d + hv].view(hk, rep, K)
            aw = w[2 * C + 2 * hv * d + hv:].view(hk, rep, K)
            t[p + "linear_attn.in_proj_qkvz.weight"] = torch.cat([qw, kw, vw, zw], 1).reshape(-1, K).bfloat16()
            t[p + "linear_attn.in_proj_ba.weight"] = torch.cat([bw, aw], 1).reshape(-1, K).bfloat16()
            t[p + "linear_attn.conv1d.weight"] = lay["conv_w"].view(-1, 1, cfg.conv_width)
            t[p + "linear_attn.A_log"] = lay["A_log"]
            t[p + "linear_attn.dt_bias"] = lay["dt_bias"]
            t[p + "linear_attn.norm.weight"] = lay["gdn_norm"]
            t[p + "linear_attn.out_proj.weight"] = _dense(lay["w_out"]).bfloat16()
        if "w_gate" in lay:
            for k, hf in (("w_gate", "gate_proj"), ("w_up", "up_proj"), ("w_down", "down_proj")):
                t[p + f"mlp.{hf}.weight"] = _dense(lay[k]).bfloat16()
        elif "router" in lay:
            t[p + "mlp.gate.weight"] = lay["router"].w
            E, I, H = cfg.moe_experts, cfg.moe_ffn, cfg.hidden
            G, U, Dn = _dense(lay["e_gate"]).view(E, I, H), _dense(lay["e_up"]).view(E, I, H), _dense(lay["e_down"]).view(E, H, I)
            for e in range(E):
                t[p + f"mlp.experts.{e}.gate_proj.weight"] = G[e].bfloat16()
                t[p + f"mlp.experts.{e}.up_proj.weight"] = U[e].bfloat16()
                t[p + f"mlp.experts.{e}.down_proj.weight"] = Dn[e].bfloat16()
            for k, hf in (("s_gate", "shared_expert.gate_proj"), ("s_up", "shared_expert.up_proj"),
                          ("s_down", "shared_expert.down_proj"), ("s_gvec", "shared_expert_gate")):
                t[p + f"mlp.{hf}.weight"] = lay[k].w
    t = {k: v.detach().contiguous().cpu() for k, v in t.items()}
    save_file(t, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump({"architectures": ["Qwen3NextForCausalLM"], "r9k_config": cfg.__dict__}, f, default=str)
