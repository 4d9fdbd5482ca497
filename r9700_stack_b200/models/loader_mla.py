"""Checkpoint loading for the sparse-MLA MoE classes (GLM-5.3-class ``MLAMoELM``, DeepSeek-V4-class
``DSV4LM``): Hugging Face DeepSeek-V3 / GLM-MoE layout -> this framework's device formats.

Names (below ``model.layers.{i}.``):
  * attention: ``self_attn.q_a_proj`` [q_lora, H], ``self_attn.q_a_layernorm``, ``self_attn.q_b_proj``
    [heads (nope + rope), q_lora], ``self_attn.kv_a_proj_with_mqa`` [kv_lora + rope, H],
    ``self_attn.kv_a_layernorm``, ``self_attn.kv_b_proj`` [heads (nope + v), kv_lora] (split per head
    into the absorbed W_uk [heads, kv_lora, nope] and W_uv [heads, v, kv_lora]), ``self_attn.o_proj``;
  * lightning indexer: ``self_attn.indexer.wq_b`` [index_heads 128, q_lora], ``self_attn.indexer.wk``
    [128, H], ``self_attn.indexer.k_norm``, ``self_attn.indexer.weights_proj`` [index_heads, H];
  * FFN: dense ``mlp.{gate,up,down}_proj`` for the first layers, else ``mlp.gate`` (router) with
    ``mlp.gate.e_score_correction_bias``, ``mlp.experts.{e}.{gate,up,down}_proj`` and
    ``mlp.shared_experts.{gate,up,down}_proj``;
  * DeepSeek-V4 class, in addition: trellis experts as ``mlp.experts.{e}.{gate,up,down}_proj.
    {trellis,suh,svh}`` (EXL3 tensor set, ``quant/exl3.py``), hyper-connection parameters
    ``hc_attn.{fn,scale,base}`` / ``hc_ffn.{...}`` and the head's ``model.hc_head.{...}``, Engram
    projections ``engram.{proj,gate}`` (the tables themselves are host-resident, loaded separately).
Linear weights may be bf16, block fp8 (``weight_scale_inv``) or NVFP4 (compressed-tensors names); the
experts convert to the model's expert format at load. Tensor-parallel ranks cut their heads, FFN
columns and experts while loading. ``dry_run`` maps every tensor name without reading data.
Reference: r9700_vllm/models/deepseek_v41_exl3.py:97-194 (name classifier, loader), :417 (dry run),
r9700_vllm/models/glm5next.py (GLM layout on stock vLLM).
"""
from __future__ import annotations

import json
import os
import re

import torch

from ..ops import linear as L
from .loader import _float_weight, _linear_stem, _Reader, index

_LAYER = re.compile(r"^model\.layers\.(\d+)\.(.+)$")
_HC = ("fn", "scale", "base")


def layer_targets(cfg, i: int, dsv4: bool = False) -> list[str]:
    """HF stems (below model.layers.{i}.) a layer of this config reads."""
    t = ["input_layernorm", "post_attention_layernorm", "self_attn.q_a_proj", "self_attn.q_a_layernorm",
         "self_attn.q_b_proj", "self_attn.kv_a_proj_with_mqa", "self_attn.kv_a_layernorm", "self_attn.kv_b_proj",
         "self_attn.o_proj", "self_attn.indexer.wq_b", "self_attn.indexer.wk", "self_attn.indexer.k_norm",
         "self_attn.indexer.weights_proj"]
    if i < cfg.first_dense:
        t += ["mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"]
    else:
        t += ["mlp.gate", "mlp.gate.e_score_correction_bias"]
        t += [f"mlp.experts.{e}.{p}" for e in range(cfg.moe_experts) for p in ("gate_proj", "up_proj", "down_proj")]
        if cfg.moe_shared_ffn:
            t += ["mlp.shared_experts.gate_proj", "mlp.shared_experts.up_proj", "mlp.shared_experts.down_proj"]
    if dsv4:
        t += [f"hc_attn.{k}" for k in _HC] + [f"hc_ffn.{k}" for k in _HC]
        if i in cfg.engram_layers:
            t += ["engram.proj", "engram.gate"]
    return t


def _stem_of(name: str) -> str:
    st = _linear_stem(name)
    if st:
        return st[0]
    for suf in (".trellis", ".suh", ".svh"):
        if name.endswith(suf):
            return name[: -len(suf)]
    return name


def dry_run(path: str, cfg, dsv4: bool = False) -> dict:
    """Map every checkpoint tensor to a model slot without reading data."""
    idx = index(path)
    top = {"model.embed_tokens", "model.norm", "lm_head"} | ({f"model.hc_head.{k}" for k in _HC} if dsv4 else set())
    expected = set(top)
    per_layer = {i: set(layer_targets(cfg, i, dsv4)) for i in range(cfg.layers)}
    for i, ts in per_layer.items():
        expected |= {f"model.layers.{i}.{s}" for s in ts}
    seen, unmapped = set(), []
    for name in idx:
        stem = _stem_of(name)
        m = _LAYER.match(stem)
        if stem in top or (m and m.group(2) in per_layer.get(int(m.group(1)), ())):
            seen.add(stem)
        else:
            unmapped.append(name)
    return {"tensors": len(idx), "mapped": len(idx) - len(unmapped), "unmapped": unmapped,
            "missing": sorted(expected - seen)}


def _vec(rd: _Reader, name: str, dev) -> torch.Tensor:
    n = name if rd.has(name) else name + ".weight"
    return rd.get(n)


def load_into(model, path: str) -> dict:
    """Overwrite a constructed MLAMoELM / DSV4LM's weights with a checkpoint's. Returns stats."""
    from .weights import from_float

    cfg, par, dev = model.cfg, model.par, model.device
    dsv4 = hasattr(model, "hc_head")
    rd = _Reader(path)
    tp, r = par.tp_size, par.tp_rank
    nh, h0 = model.nh, r * model.nh
    QH, LAT = cfg.qk_nope + 64, None
    bf = lambda t: L.BF16Weight(t.to(dev, torch.bfloat16).contiguous())  # noqa: E731
    model.embed = rd.get("model.embed_tokens.weight").to(dev, torch.bfloat16)
    model.final_norm = rd.get("model.norm.weight").to(dev, torch.bfloat16)
    vl = model.vocab_local
    model.lm_head = bf(_float_weight(rd, "lm_head", dev)[r * vl:(r + 1) * vl])
    for i, lay in enumerate(model.layers):
        p = f"model.layers.{i}."
        g = lambda s: _float_weight(rd, p + s, dev)  # noqa: E731
        lay["in_norm"] = _vec(rd, p + "input_layernorm", dev).to(dev, torch.bfloat16)
        lay["post_norm"] = _vec(rd, p + "post_attention_layernorm", dev).to(dev, torch.bfloat16)
        lay["w_dq"] = bf(g("self_attn.q_a_proj"))
        lay["q_norm"] = _vec(rd, p + "self_attn.q_a_layernorm", dev).to(dev, torch.bfloat16)
        lay["w_uq"] = bf(g("self_attn.q_b_proj")[h0 * QH:(h0 + nh) * QH])
        lay["w_dkv"] = bf(g("self_attn.kv_a_proj_with_mqa"))
        lay["kv_norm"] = _vec(rd, p + "self_attn.kv_a_layernorm", dev).to(dev, torch.bfloat16)
        kvb = g("self_attn.kv_b_proj")
        LAT = kvb.shape[1]
        kvb = kvb.view(cfg.n_heads, cfg.qk_nope + cfg.v_head, LAT)[h0:h0 + nh]
        lay["w_uk"] = kvb[:, : cfg.qk_nope].transpose(1, 2).to(torch.bfloat16).contiguous()  # [nh, LAT, nope]
        lay["w_uv"] = kvb[:, cfg.qk_nope:].to(torch.bfloat16).contiguous()  # [nh, v, LAT]
        lay["w_o"] = bf(g("self_attn.o_proj")[:, h0 * cfg.v_head:(h0 + nh) * cfg.v_head])
        lay["w_iq"] = bf(g("self_attn.indexer.wq_b"))
        lay["w_ik"] = bf(g("self_attn.indexer.wk"))
        lay["ik_norm"] = _vec(rd, p + "self_attn.indexer.k_norm", dev).to(dev, torch.bfloat16)
        lay["w_iw"] = bf(g("self_attn.indexer.weights_proj"))
        if i < cfg.first_dense:
            dl = model.dense_local
            lay["w_gate"] = bf(g("mlp.gate_proj")[r * dl:(r + 1) * dl])
            lay["w_up"] = bf(g("mlp.up_proj")[r * dl:(r + 1) * dl])
            lay["w_down"] = bf(g("mlp.down_proj")[:, r * dl:(r + 1) * dl])
        else:
            El, e0 = model.e_local, r * model.e_local
            lay["router"] = bf(g("mlp.gate"))
            lay["router_bias"] = _vec(rd, p + "mlp.gate.e_score_correction_bias", dev).float().to(dev)
            if getattr(model, "mx_experts", True):
                for key, hf in (("e_gate", "gate_proj"), ("e_up", "up_proj"), ("e_down", "down_proj")):
                    ws = torch.cat([g(f"mlp.experts.{e}.{hf}") for e in range(e0, e0 + El)], 0)
                    lay[key] = from_float(ws.contiguous(), cfg.expert_format, tiled=True)
            else:
                from ..ops import exl3 as X

                for key, hf in (("x_gate", "gate_proj"), ("x_up", "up_proj"), ("x_down", "down_proj")):
                    st = [p + f"mlp.experts.{e}.{hf}" for e in range(e0, e0 + El)]
                    tr = torch.stack([rd.get(s + ".trellis") for s in st]).to(dev)
                    lay[key] = X.Exl3Linear(tr.contiguous(), torch.stack([rd.get(s + ".suh") for s in st]).to(dev),
                                            torch.stack([rd.get(s + ".svh") for s in st]).to(dev),
                                            tr.shape[-1] // 16, lay[key].cb if key in lay else 1)
            if model.shared_local:
                sl = model.shared_local
                lay["s_gate"] = bf(g("mlp.shared_experts.gate_proj")[r * sl:(r + 1) * sl])
                lay["s_up"] = bf(g("mlp.shared_experts.up_proj")[r * sl:(r + 1) * sl])
                lay["s_down"] = bf(g("mlp.shared_experts.down_proj")[:, r * sl:(r + 1) * sl])
        if dsv4:
            for hk in ("hc_attn", "hc_ffn"):
                prm = lay[hk]
                for k in _HC:
                    getattr(prm, k).copy_(rd.get(p + f"{hk}.{k}").to(dev))
            if "eng_proj" in lay:
                lay["eng_proj"] = bf(g("engram.proj"))
                lay["eng_gate"] = bf(g("engram.gate"))
    if dsv4:
        for k in _HC:
            getattr(model.hc_head, k).copy_(rd.get(f"model.hc_head.{k}").to(dev))
    return {"layers": len(model.layers), "kv_lora": LAT}


def export_hf(model, path: str) -> None:
    """Write a single-rank MLA / DeepSeek-class model in the layout above (bf16, trellis tensors as
    stored), for round-trip tests and for handing a synthetic model on."""
    from safetensors.torch import save_file

    from .loader import _dense

    assert model.par.tp_size == 1
    cfg = model.cfg
    dsv4 = hasattr(model, "hc_head")
    os.makedirs(path, exist_ok=True)
    t = {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.final_norm,
         "lm_head.weight": _dense(model.lm_head).bfloat16()}
    for i, lay in enumerate(model.layers):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = lay["in_norm"]
        t[p + "post_attention_layernorm.weight"] = lay["post_norm"]
        for k, hf in (("w_dq", "self_attn.q_a_proj"), ("w_uq", "self_attn.q_b_proj"),
                      ("w_dkv", "self_attn.kv_a_proj_with_mqa"), ("w_o", "self_attn.o_proj"),
                      ("w_iq", "self_attn.indexer.wq_b"), ("w_ik", "self_attn.indexer.wk"),
                      ("w_iw", "self_attn.indexer.weights_proj")):
            t[p + hf + ".weight"] = _dense(lay[k]).bfloat16()
        t[p + "self_attn.q_a_layernorm.weight"] = lay["q_norm"]
        t[p + "self_attn.kv_a_layernorm.weight"] = lay["kv_norm"]
        t[p + "self_attn.indexer.k_norm.weight"] = lay["ik_norm"]
        uk = lay["w_uk"].float().transpose(1, 2)  # [nh, nope, LAT]
        t[p + "self_attn.kv_b_proj.weight"] = torch.cat([uk, lay["w_uv"].float()], 1).reshape(-1, uk.shape[-1]).bfloat16()
        if "w_gate" in lay:
            for k, hf in (("w_gate", "gate_proj"), ("w_up", "up_proj"), ("w_down", "down_proj")):
                t[p + f"mlp.{hf}.weight"] = _dense(lay[k]).bfloat16()
        else:
            t[p + "mlp.gate.weight"] = lay["router"].w
            t[p + "mlp.gate.e_score_correction_bias"] = lay["router_bias"]
            E, I, H = cfg.moe_experts, cfg.moe_ffn, cfg.hidden
            if "e_gate" in lay:
                G, U = _dense(lay["e_gate"]).view(E, I, H), _dense(lay["e_up"]).view(E, I, H)
                Dn = _dense(lay["e_down"]).view(E, H, I)
                for e in range(E):
                    t[p + f"mlp.experts.{e}.gate_proj.weight"] = G[e].bfloat16()
                    t[p + f"mlp.experts.{e}.up_proj.weight"] = U[e].bfloat16()
                    t[p + f"mlp.experts.{e}.down_proj.weight"] = Dn[e].bfloat16()
            else:
                for key, hf in (("x_gate", "gate_proj"), ("x_up", "up_proj"), ("x_down", "down_proj")):
                    x = lay[key]
                    for e in range(E):
                        t[p + f"mlp.experts.{e}.{hf}.trellis"] = x.trellis[e]
                        t[p + f"mlp.experts.{e}.{hf}.suh"] = x.suh[e]
                        t[p + f"mlp.experts.{e}.{hf}.svh"] = x.svh[e]
            if "s_gate" in lay:
                for k, hf in (("s_gate", "gate_proj"), ("s_up", "up_proj"), ("s_down", "down_proj")):
                    t[p + f"mlp.shared_experts.{hf}.weight"] = lay[k].w
        if dsv4:
            for hk in ("hc_attn", "hc_ffn"):
                for k in _HC:
                    t[p + f"{hk}.{k}"] = getattr(lay[hk], k)
            if "eng_proj" in lay:
                t[p + "engram.proj.weight"] = lay["eng_proj"].w
                t[p + "engram.gate.weight"] = lay["eng_gate"].w
    if dsv4:
        for k in _HC:
            t[f"model.hc_head.{k}"] = getattr(model.hc_head, k)
    t = {k: v.detach().contiguous().cpu() for k, v in t.items()}
    save_file(t, os.path.join(path, "model.safetensors"))
    arch = "DeepseekV3ForCausalLM" if not dsv4 else "DeepseekV4ForCausalLM"
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump({"architectures": [arch], "r9k_config": cfg.__dict__}, f, default=str)
