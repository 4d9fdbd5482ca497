"""Serving end to end on a B200: HTTP requests through the async engine on the tiny hybrid model
give the same tokens as LLM.generate, concurrently; sampled requests are reproducible per seed."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_server_matches_generate():
    from fastapi.testclient import TestClient

    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_hybrid
    from r9700_stack_b200.serve.async_engine import AsyncEngine
    from r9700_stack_b200.serve.openai_server import build_app
    from r9700_stack_b200.serve.tokenizer import ByteTokenizer

    cfg = tiny_hybrid()
    ec = EngineConfig(max_batch=4, max_model_len=512, max_prefill_tokens=128, graph_batch_sizes=[1, 2, 4])
    prompts = [[5, 6, 7, 8, 9], list(range(20, 90)), [300, 301]]
    ref = LLM(cfg, ec, seed=3).generate(prompts, SamplingParams(max_tokens=12))
    torch.cuda.synchronize()
    eng = AsyncEngine(LLM(cfg, ec, seed=3))
    eng.start()
    app = build_app(eng, ByteTokenizer(cfg.vocab), "tiny", ec.max_model_len)
    try:
        with TestClient(app) as c:
            import concurrent.futures as cf

            def ask(p):
                return c.post("/v1/completions", json={"prompt": p, "max_tokens": 12, "ignore_eos": True}).json()

            with cf.ThreadPoolExecutor(3) as ex:
                outs = list(ex.map(ask, prompts))
            for o, r in zip(outs, ref):
                assert o["choices"][0]["token_ids"] == r
            s1 = c.post("/v1/completions", json={"prompt": prompts[0], "max_tokens": 8, "temperature": 1.0,
                                                  "seed": 11, "ignore_eos": True}).json()
            s2 = c.post("/v1/completions", json={"prompt": prompts[0], "max_tokens": 8, "temperature": 1.0,
                                                  "seed": 11, "ignore_eos": True}).json()
            assert s1["choices"][0]["token_ids"] == s2["choices"][0]["token_ids"]
            assert len(s1["choices"][0]["token_ids"]) == 8
    finally:
        eng.stop()
    from r9700_stack_b200.utils import status

    status.check()
