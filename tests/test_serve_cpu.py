"""Serving front end on CPU: OpenAI-compatible endpoints, streaming, aborts and metrics over the
async engine, driven by a fake engine with the LLM interface (no GPU)."""
import asyncio
import json

import pytest
import torch

from r9700_stack_b200.engine.scheduler import SamplingParams, Sequence
from r9700_stack_b200.serve.async_engine import AsyncEngine
from r9700_stack_b200.serve.tokenizer import ByteTokenizer


class FakeLLM:
    """Emits token (last + 1) % 259 + 3 per step for every running request; two tokens per step when
    ``burst`` (as a speculative step would)."""

    def __init__(self, burst=1):
        self.running: list[Sequence] = []
        self.burst = burst
        self.spec_stats = {"steps": 0, "drafted": 0, "accepted": 0}

    def add_request(self, prompt, params):
        s = Sequence(list(prompt), params)
        self.running.append(s)
        return s

    def abort(self, seq):
        if seq in self.running:
            self.running.remove(seq)
        seq.finished = True

    def has_unfinished(self):
        return bool(self.running)

    def step(self):
        for s in list(self.running):
            for _ in range(self.burst):
                t = (s.tokens[-1] + 1) % 256 + 3
                s.output.append(t)
                if len(s.output) >= s.params.max_tokens or (not s.params.ignore_eos and t == s.params.eos_token_id):
                    s.finished = True
                    self.running.remove(s)
                    break


@pytest.fixture()
def client():
    from fastapi.testclient import TestClient

    from r9700_stack_b200.serve.openai_server import build_app

    eng = AsyncEngine(FakeLLM(burst=2))
    eng.start()
    app = build_app(eng, ByteTokenizer(512), "fake", 4096)
    with TestClient(app) as c:
        yield c, eng
    eng.stop()


def test_models_health(client):
    c, _ = client
    assert c.get("/health").json()["status"] == "ok"
    assert c.get("/v1/models").json()["data"][0]["id"] == "fake"


def test_completion_text_and_ids(client):
    c, _ = client
    r = c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 5})
    assert r.status_code == 200
    d = r.json()
    toks = d["choices"][0]["token_ids"]
    # 'b' = 98 -> id 101; then (101+1)%256+3 = 105, ...
    assert toks == [105, 109, 113, 117, 121]
    assert d["usage"] == {"prompt_tokens": 2, "completion_tokens": 5, "total_tokens": 7}
    assert d["choices"][0]["finish_reason"] == "length"
    r = c.post("/v1/completions", json={"prompt": [10, 20], "max_tokens": 3})
    assert r.json()["choices"][0]["token_ids"] == [24, 28, 32]


def test_completion_stream(client):
    c, _ = client
    with c.stream("POST", "/v1/completions", json={"prompt": [10], "max_tokens": 7, "stream": True}) as r:
        lines = [l for l in r.iter_lines() if l.startswith("data:")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(l[5:]) for l in lines[:-1]]
    toks = [t for ch in chunks for c0 in ch["choices"] for t in c0["token_ids"]]
    assert toks == [14, 18, 22, 26, 30, 34, 38]
    assert chunks[-1]["usage"]["completion_tokens"] == 7


def test_chat(client):
    c, _ = client
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4})
    d = r.json()
    assert d["object"] == "chat.completion" and d["choices"][0]["message"]["role"] == "assistant"
    assert d["usage"]["completion_tokens"] == 4


def test_errors(client):
    c, _ = client
    assert c.post("/v1/completions", json={"prompt": [], "max_tokens": 4}).status_code == 400
    assert c.post("/v1/completions", json={"prompt": [99999], "max_tokens": 4}).status_code == 400
    assert c.post("/v1/completions", json={"prompt": "x", "max_tokens": 0}).status_code == 400
    assert c.post("/v1/completions", json={"prompt": "x", "max_tokens": 5000}).status_code == 400


def test_metrics(client):
    c, _ = client
    c.post("/v1/completions", json={"prompt": [5], "max_tokens": 4})
    m = c.get("/metrics").text
    assert "r9k_generation_tokens_total 4" in m and "r9k_requests_finished_total 1" in m


def test_concurrent_requests_and_abort():
    eng = AsyncEngine(FakeLLM())
    eng.start()

    async def run():
        async def full(p, n):
            toks = []
            async for o in eng.generate(p, SamplingParams(max_tokens=n)):
                toks += o.new_tokens
            return toks

        async def aborted():
            got = 0
            async for o in eng.generate([7], SamplingParams(max_tokens=10_000)):
                got += len(o.new_tokens)
                if got >= 3:
                    break
            return got

        return await asyncio.gather(full([1], 6), full([2], 3), aborted())

    a, b, n = asyncio.run(run())
    assert len(a) == 6 and len(b) == 3 and n >= 3
    import time

    for _ in range(100):
        if not eng.llm.running:
            break
        time.sleep(0.01)
    assert not eng.llm.running  # the aborted request was dropped
    eng.stop()


def test_sampler_cpu():
    from r9700_stack_b200.engine.sampler import sample_rows

    torch.manual_seed(0)
    logits = torch.randn(4, 50)
    g = SamplingParams(temperature=0)
    t1 = SamplingParams(temperature=1.0, top_k=1)
    tp = SamplingParams(temperature=1.0, top_p=1e-6)
    hot = SamplingParams(temperature=1.0, seed=5)
    out = sample_rows(logits, [g, t1, tp, hot], [0, 0, 0, 3])
    am = logits.argmax(-1).tolist()
    assert out[:3] == am[:3]
    assert out[3] == sample_rows(logits, [g, g, g, hot], [0, 0, 0, 3])[3]  # seeded per request/step
    draws = [sample_rows(logits[3:4], [SamplingParams(temperature=1.0, seed=s)], [0])[0] for s in range(400)]
    p = torch.softmax(logits[3], -1)
    top = int(p.argmax())
    assert abs(draws.count(top) / 400 - float(p[top])) < 0.08


def test_launch_dry_run(capsys):
    from r9700_stack_b200.serve.launch import main

    assert main(["--model", "dense27b", "--dry-run", "--spec", "block"]) == 0
    d = json.loads(capsys.readouterr().out)
    assert d["engine"]["spec_tokens"] == 7 and d["kv_cache_gb_per_rank"] > 0
