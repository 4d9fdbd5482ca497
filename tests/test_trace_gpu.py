"""Device trace marks inside eager forwards and decode graph replays, and the profiler step ledger."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_device_trace_eager_and_graph():
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_hybrid
    from r9700_stack_b200.utils.trace import DeviceTrace, step_ledger

    cfg = tiny_hybrid()
    ec = EngineConfig(max_batch=2, max_model_len=512, max_prefill_tokens=256, cuda_graphs=True, graph_batch_sizes=[1, 2])
    llm = LLM(cfg, ec, seed=1)
    tr = DeviceTrace(llm.model.device)
    llm.model.trace = tr
    llm.runner.capture_decode_graphs()  # recapture with the marks inside the graphs
    llm.add_request(list(range(1, 40)), SamplingParams(max_tokens=8))
    llm.step()  # eager prefill
    rows = tr.read()
    assert [n for n, _ in rows][:2] == ["L0.gdn", "L0.ffn"] and rows[-1][0] == "lm_head"
    assert all(us >= 0 for _, us in rows)
    llm.step()  # decode: graph replay writes the same marks
    s = tr.summary()
    assert s["total_us"] > 0 and {"attn", "gdn", "ffn", "lm_head"} <= set(s)
    led = step_ledger(llm, steps=3)
    assert led["kernel_ms_per_step"] > 0 and "gemm_tcgen05" in led["by_family_ms_per_step"]
