"""Checkpoint loader of the sparse-MLA MoE classes: the name-mapping dry run on a synthetic
DeepSeek-V3 / GLM-MoE layout (CPU, also with the DeepSeek-V4 trellis / hyper-connection names), and a
round trip export -> load into a differently seeded model that reproduces its logits (GPU)."""
import pytest
import torch


def _fake_ckpt(path, cfg, dsv4=False):
    from safetensors.torch import save_file

    from r9700_stack_b200.models.loader_mla import layer_targets

    t = {"model.embed_tokens.weight": torch.zeros(1), "model.norm.weight": torch.zeros(1),
         "lm_head.weight": torch.zeros(1)}
    if dsv4:
        t.update({f"model.hc_head.{k}": torch.zeros(1) for k in ("fn", "scale", "base")})
    for i in range(cfg.layers):
        for stem in layer_targets(cfg, i, dsv4):
            if dsv4 and ".experts." in stem:
                for suf in ("trellis", "suh", "svh"):
                    t[f"model.layers.{i}.{stem}.{suf}"] = torch.zeros(1)
            elif stem.endswith(("e_score_correction_bias", ".fn", ".scale", ".base")):
                t[f"model.layers.{i}.{stem}"] = torch.zeros(1)
            else:
                t[f"model.layers.{i}.{stem}.weight"] = torch.zeros(1)
    t["model.layers.0.self_attn.rotary_emb.inv_freq"] = torch.zeros(1)
    save_file(t, str(path / "model.safetensors"))


@pytest.mark.parametrize("dsv4", [False, True])
def test_dry_run_maps_names(tmp_path, dsv4):
    from r9700_stack_b200.models.dsv4 import tiny_dsv4
    from r9700_stack_b200.models.loader_mla import dry_run
    from r9700_stack_b200.models.mla_moe import tiny_mla

    cfg = tiny_dsv4() if dsv4 else tiny_mla()
    _fake_ckpt(tmp_path, cfg, dsv4)
    r = dry_run(str(tmp_path), cfg, dsv4=dsv4)
    assert r["unmapped"] == ["model.layers.0.self_attn.rotary_emb.inv_freq"]
    assert r["missing"] == []


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["mla", "dsv4"])
def test_export_load_roundtrip(tmp_path, name):
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig
    from r9700_stack_b200.models.dsv4 import tiny_dsv4
    from r9700_stack_b200.models.loader_mla import dry_run, export_hf, load_into
    from r9700_stack_b200.models.mla_moe import tiny_mla

    cfg = tiny_dsv4() if name == "dsv4" else tiny_mla()
    ec = EngineConfig(max_batch=2, max_model_len=128, max_prefill_tokens=64, cuda_graphs=False)
    a = LLM(cfg, ec, seed=1)
    export_hf(a.model, str(tmp_path))
    assert dry_run(str(tmp_path), cfg, dsv4=name == "dsv4")["missing"] == []
    b = LLM(cfg, ec, seed=2)  # different random weights, then the checkpoint's
    load_into(b.model, str(tmp_path))
    for la_, lb_ in zip(a.model.layers, b.model.layers):
        if "engram" in la_:
            lb_["engram"] = la_["engram"]  # host-resident tables load separately from the shards
    p = [list(range(3, 40))]
    a.generate(p, SamplingParams(max_tokens=3))
    la = a.runner.ws.logits[0].clone()
    b.generate(p, SamplingParams(max_tokens=3))
    lb = b.runner.ws.logits[0].clone()
    # NVFP4 experts are re-quantised from their exported values (close, not bit-equal); trellis
    # experts and bf16 tensors round-trip exactly
    cos = torch.nn.functional.cosine_similarity(la.double(), lb.double(), dim=0)
    assert float(cos) > 0.999, float(cos)
