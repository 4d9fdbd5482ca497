"""Checkpoint loader: the name-mapping dry run on a synthetic HF-layout checkpoint (CPU), and a
round trip export -> load that reproduces the model's logits (GPU)."""
import pytest
import torch


def _fake_ckpt(path, cfg):
    """Zero-filled tensors with the HF names and shapes of a tiny hybrid config."""
    from safetensors.torch import save_file

    from r9700_stack_b200.models.loader import layer_targets

    H, d = cfg.hidden, cfg.gdn_head_dim
    t = {"model.embed_tokens.weight": torch.zeros(cfg.vocab, H), "model.norm.weight": torch.zeros(H),
         "lm_head.weight": torch.zeros(cfg.vocab, H)}
    for i in range(cfg.layers):
        for stem in layer_targets(cfg, i):
            t[f"model.layers.{i}.{stem}.weight" if not stem.endswith(("A_log", "dt_bias")) else
              f"model.layers.{i}.{stem}"] = torch.zeros(1)
    t["model.layers.0.unexpected.weight"] = torch.zeros(1)
    save_file(t, str(path / "model.safetensors"))


def test_dry_run_maps_names(tmp_path):
    from r9700_stack_b200.models.config import tiny_hybrid
    from r9700_stack_b200.models.loader import dry_run

    cfg = tiny_hybrid()
    _fake_ckpt(tmp_path, cfg)
    r = dry_run(str(tmp_path), cfg)
    assert r["unmapped"] == ["model.layers.0.unexpected.weight"]
    assert r["missing"] == []
    assert r["mapped"] == r["tensors"] - 1


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny_hybrid", "tiny_moe"])
def test_export_load_roundtrip(tmp_path, name):
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models import config as C
    from r9700_stack_b200.models.config import EngineConfig
    from r9700_stack_b200.models.loader import dry_run, export_hf, load_into

    cfg = getattr(C, name)(weight_format="bf16", lm_head_format="bf16")
    ec = EngineConfig(max_batch=2, max_model_len=128, max_prefill_tokens=64, cuda_graphs=False)
    a = LLM(cfg, ec, seed=1)
    export_hf(a.model, str(tmp_path))
    assert dry_run(str(tmp_path), cfg)["missing"] == []
    b = LLM(cfg, ec, seed=2)  # different random weights, then the checkpoint's
    load_into(b.model, str(tmp_path))
    p = [list(range(3, 40))]
    ra = a.generate(p, SamplingParams(max_tokens=5))
    la = a.runner.ws.logits[0].clone()
    rb = b.generate(p, SamplingParams(max_tokens=5))
    lb = b.runner.ws.logits[0].clone()
    if name == "tiny_hybrid":
        # bf16 weights round-trip exactly
        assert ra == rb
        torch.testing.assert_close(la, lb, rtol=0, atol=0)
    else:
        # MXFP4 experts are re-quantised from their exported values: close, not bit-equal
        cos = torch.nn.functional.cosine_similarity(la.double(), lb.double(), dim=0)
        assert float(cos) > 0.999, float(cos)
