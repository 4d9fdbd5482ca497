"""Sparse-MLA MoE model (tiny GLM-class) vs its PyTorch oracle, through the engine (prefill, graph
decode), with a context longer than the indexer's top-k so the selection is exercised."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_tiny_mla_matches_reference():
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig
    from r9700_stack_b200.models.mla_moe import tiny_mla
    from r9700_stack_b200.models.reference_mla import MLARefState, reference_forward_mla
    from r9700_stack_b200.utils import status

    cfg = tiny_mla()
    ec = EngineConfig(max_batch=2, max_model_len=256, max_prefill_tokens=64, graph_batch_sizes=[1, 2])
    llm = LLM(cfg, ec, seed=5)
    prompt = list(range(7, 37))  # 30 tokens > index_topk 24
    seq = llm.add_request(prompt, SamplingParams(max_tokens=4))
    st = MLARefState(llm.model)
    llm.step()
    torch.cuda.synchronize()
    status.check()
    got = llm.runner.ws.logits[0].clone()
    ref = reference_forward_mla(llm.model, prompt, st)[-1]
    cos = torch.nn.functional.cosine_similarity(got.double(), ref.double(), dim=0)
    assert float(cos) > 0.99, float(cos)
    for _ in range(2):
        llm.step()
        torch.cuda.synchronize()
        got = llm.runner.ws.logits[0].clone()
        ref = reference_forward_mla(llm.model, [seq.output[-2]], st)[-1]
        cos = torch.nn.functional.cosine_similarity(got.double(), ref.double(), dim=0)
        assert float(cos) > 0.99, float(cos)
    status.check()


def test_tiny_mla_generate_graph_equals_eager():
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig
    from r9700_stack_b200.models.mla_moe import tiny_mla

    outs = []
    for graphs in (False, True):
        ec = EngineConfig(max_batch=3, max_model_len=256, max_prefill_tokens=64, cuda_graphs=graphs,
                          graph_batch_sizes=[1, 2, 4])
        llm = LLM(tiny_mla(), ec, seed=2)
        outs.append(llm.generate([[5, 6, 7], list(range(40, 80)), [9] * 30], SamplingParams(max_tokens=6)))
    assert outs[0] == outs[1]
