"""Serving release gates on CPU over the async engine with a fake LLM: a correct engine passes
stress and a short soak; engines that drop tokens, diverge on duplicates or leak KV blocks fail."""
import asyncio

from r9700_stack_b200.engine.cache import BlockAllocator, SlotAllocator
from r9700_stack_b200.engine.scheduler import Sequence
from r9700_stack_b200.serve import gates
from r9700_stack_b200.serve.async_engine import AsyncEngine


class _Sched:
    def __init__(self):
        self.blocks = BlockAllocator(64)
        self.slots = SlotAllocator(8)


class FakeLLM:
    """Deterministic next token = hash of the context; admits at most max_batch sequences per step."""

    def __init__(self, max_batch=4, bug=None):
        self.waiting, self.running = [], []
        self.max_batch, self.bug = max_batch, bug
        self.scheduler = _Sched()
        self._held = {}

    def add_request(self, prompt, params):
        s = Sequence(list(prompt), params)
        self.waiting.append(s)
        return s

    def abort(self, seq):
        for q in (self.waiting, self.running):
            if seq in q:
                q.remove(seq)
        self._release(seq)
        seq.finished = True

    def has_unfinished(self):
        return bool(self.waiting or self.running)

    def _release(self, s):
        b = self._held.pop(id(s), None)
        if b is not None and self.bug != "leak":
            self.scheduler.blocks.free(b)

    def step(self):
        while self.waiting and len(self.running) < self.max_batch:
            s = self.waiting.pop(0)
            self._held[id(s)] = self.scheduler.blocks.allocate(1)
            self.running.append(s)
        for i, s in enumerate(list(self.running)):
            t = (sum(s.tokens) * 31 + len(s.tokens)) % 500
            if self.bug == "diverge" and i == 1:
                t = (t + 1) % 500
            s.output.append(t)
            limit = s.params.max_tokens - (1 if self.bug == "short" else 0)
            if len(s.output) >= limit:
                s.finished = True
                self.running.remove(s)
                self._release(s)


def _run(coro_fn, llm):
    eng = AsyncEngine(llm)
    eng.start()
    try:
        return asyncio.run(coro_fn(eng))
    finally:
        eng.stop()


def test_stress_passes_and_catches_bugs():
    r = _run(lambda e: gates.stress(e, 20, 6, 512), FakeLLM())
    assert r["pass"] and r["requests"] == 20 and r["pairs"] == 10, r
    r = _run(lambda e: gates.stress(e, 20, 6, 512), FakeLLM(bug="short"))
    assert not r["pass"] and r["wrong_length"] == 20
    r = _run(lambda e: gates.stress(e, 20, 6, 512), FakeLLM(bug="diverge"))
    assert not r["pass"] and r["mismatched_pairs"] > 0
    r = _run(lambda e: gates.stress(e, 20, 6, 512, strict=False, tolerate=20), FakeLLM(bug="diverge"))
    assert r["pass"]


def test_soak_short_and_leak_detection():
    r = _run(lambda e: gates.soak(e, 0.5, 4, 512, prompt_range=(2, 20), output_range=(1, 8)), FakeLLM())
    assert r["pass"] and r["requests"] > 0 and r["kv_free_end"] == r["kv_free_start"], r
    r = _run(lambda e: gates.soak(e, 0.3, 4, 512, prompt_range=(2, 20), output_range=(1, 8)), FakeLLM(bug="leak"))
    assert not r["pass"] and r["kv_free_end"] != r["kv_free_start"]


def test_ttft_by_length():
    r = _run(lambda e: gates.ttft_by_length(e, [4, 32], 512, reps=2), FakeLLM())
    assert set(r["by_prompt_tokens"]) == {4, 32}
