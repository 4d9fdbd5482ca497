"""Hyper-connection kernels (gate_mix, combine_norm) against their torch restatements, and a tiny
hybrid model with HC residual streams against the fp32 oracle."""
import pytest
import torch

from r9700_stack_b200.ops import hc as HC

pytestmark = pytest.mark.gpu


def _check():
    from r9700_stack_b200.utils import status

    torch.cuda.synchronize()
    status.check()


@pytest.mark.parametrize("hc,hd", [(4, 256), (2, 2048), (8, 5120), (4, 8192)])
def test_gate_mix(hc, hd):
    torch.manual_seed(0)
    T = 7
    x = torch.randn(T, hc * hd).bfloat16().cuda()
    for g in (torch.randn(T, hc * hd).bfloat16().cuda(), torch.randn(1, hc * hd).bfloat16().cuda()):
        out = torch.empty(T, hd, dtype=torch.bfloat16, device="cuda")
        HC.gate_mix(x, g, hc, out)
        _check()
        ref = HC.gate_mix_ref(x, g, hc)
        assert torch.allclose(out.float(), ref.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("hc,hd", [(4, 256), (2, 2048), (8, 5120), (4, 8192)])
@pytest.mark.parametrize("per_stream", [True, False])
@pytest.mark.parametrize("with_block", [True, False])
def test_combine_norm(hc, hd, per_stream, with_block):
    torch.manual_seed(1)
    T = 5
    res = torch.randn(T, hc * hd).bfloat16().cuda()
    blk = torch.randn(T, hd).bfloat16().cuda() if with_block else None
    l = torch.randn(T, hc).cuda() if with_block else None
    w = (torch.randn(hc * hd if per_stream else hd) * 0.1).bfloat16().cuda()
    ref_res, ref_y = HC.combine_norm_ref(res.clone(), blk, l, w, hc, 1e-6)
    y = torch.empty_like(res)
    HC.combine_norm(res, blk, l, w, hc, 1e-6, y)
    _check()
    # within one bf16 rounding: the kernel's sigmoid and fused multiply-add round differently from torch's
    assert torch.allclose(res.float().cpu(), ref_res.float().cpu(), atol=1e-2, rtol=1e-2)
    assert torch.allclose(y.float(), ref_y.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("fused", ["1", "0"])
@pytest.mark.parametrize("moe", [False, True])
def test_tiny_hc_model_matches_reference(moe, fused, monkeypatch, request):
    from r9700_stack_b200 import knobs

    monkeypatch.setenv("R9K_HC_FUSED", fused)
    knobs.refresh()
    request.addfinalizer(knobs.refresh)  # runs after monkeypatch restored the environment
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_hybrid, tiny_moe
    from r9700_stack_b200.models.reference import ReferenceState, reference_forward

    cfg = (tiny_moe if moe else tiny_hybrid)(gdn_state_dtype="fp32", hc_streams=4)
    ec = EngineConfig(max_batch=2, max_model_len=512, max_prefill_tokens=256, cuda_graphs=True, graph_batch_sizes=[1, 2])
    llm = LLM(cfg, ec, seed=3)
    prompt = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(5)).tolist()
    seq = llm.add_request(prompt, SamplingParams(max_tokens=5))
    st = ReferenceState(llm.model)
    llm.step()
    _check()
    cos = lambda a, b: float(torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))
    got = llm.runner.ws.logits[0].clone()
    ref = reference_forward(llm.model, prompt, st)[-1]
    assert cos(got, ref) > 0.995, cos(got, ref)
    for _ in range(4):
        llm.step()
        _check()
        got = llm.runner.ws.logits[0].clone()
        ref = reference_forward(llm.model, [seq.output[-2]], st)[-1]
        assert cos(got, ref) > 0.99, cos(got, ref)


@pytest.mark.parametrize("hc,hd", [(4, 2048), (2, 5120), (8, 256)])
@pytest.mark.parametrize("with_block", [True, False])
def test_fused_point(hc, hd, with_block):
    from r9700_stack_b200.models.weights import WeightFactory

    torch.manual_seed(2)
    T = 6
    p = HC.random_point(WeightFactory(torch.device("cuda"), seed=5, std=0.02), hc, hd)
    res = torch.randn(T, hc * hd).bfloat16().cuda()
    y = torch.randn(T, hd).bfloat16().cuda() if with_block else None
    ref_res, ref_out = HC.point_ref(res.clone(), y, p, hc, 1e-6)
    out = torch.empty(T, hd, dtype=torch.bfloat16, device="cuda")
    HC.point(res, y, p, hc, 1e-6, out)
    _check()
    assert torch.allclose(res.float(), ref_res.float(), atol=1e-2, rtol=1e-2)
    assert torch.allclose(out.float(), ref_out.float(), atol=2e-2, rtol=2e-2)
