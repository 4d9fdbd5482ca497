"""Serving release gates, run in process over the async engine (the real ``LLM`` or any object with
its interface): the roles of the reference's bench/sanity_stress.py (strict sanity above the batch
limit), bench/soak.py (mixed-length soak), bench/itl.py and bench/ttft_breakdown.py.

    python -m r9700_stack_b200.serve.gates stress --model tiny-hybrid --requests 48 --max-batch 16
    python -m r9700_stack_b200.serve.gates soak --model dense27b --seconds 900 --concurrency 24
    python -m r9700_stack_b200.serve.gates ttft --model dense27b --lengths 128,1024,8192

Every gate returns a dict with ``"pass"`` and the figures it judged; the CLI prints it as one JSON line
and exits non-zero on failure.

* stress: more concurrent requests than the engine's batch limit, every prompt submitted twice.
  Passes when every request finishes with exactly ``max_tokens`` in-vocabulary tokens and the two
  copies of each prompt produce the same greedy tokens (``strict``) or at most ``tolerate`` pairs differ.
* soak: keeps ``concurrency`` requests of random prompt and output lengths in flight for ``seconds``.
  Passes when nothing errors, every request finishes with its length, the engine drains, and the
  KV blocks and (on a GPU) the allocated device memory return to their starting values.
* ttft / itl: time to first token by prompt length, inter-token latency percentiles.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import statistics
import sys
import time

from ..engine.scheduler import SamplingParams


def _pct(xs: list[float], p: float) -> float | None:
    if not xs:
        return None
    ys = sorted(xs)
    return ys[min(len(ys) - 1, int(round(p / 100 * (len(ys) - 1))))]


async def _run_one(engine, prompt: list[int], max_tokens: int) -> dict:
    params = SamplingParams(max_tokens=max_tokens, temperature=0.0, ignore_eos=True)
    t0 = time.perf_counter()
    toks, stamps, reason = [], [], None
    async for out in engine.generate(prompt, params):
        now = time.perf_counter()
        if out.new_tokens:
            toks.extend(out.new_tokens)
            stamps.extend([now] * len(out.new_tokens))
        if out.finished:
            reason = out.finish_reason
    if reason == "error":
        raise RuntimeError(f"engine step failed: {getattr(engine.metrics, 'last_error', None)}")
    ttft = stamps[0] - t0 if stamps else None
    itl = [b - a for a, b in zip(stamps, stamps[1:]) if b > a]
    return {"tokens": toks, "ttft_s": ttft, "itl_s": itl, "reason": reason, "total_s": time.perf_counter() - t0}


def _kv_free(llm) -> tuple | None:
    """(free KV blocks, free state slots) of the engine's scheduler, when it has one."""
    sched = getattr(llm, "scheduler", None)
    if sched is None or not hasattr(sched, "blocks"):
        return None
    return (sched.blocks.num_free, sched.slots.num_free)


def _device_bytes() -> int | None:
    try:
        import torch

        if torch.cuda.is_available():
            torch.cuda.synchronize()
            return int(torch.cuda.memory_allocated())
    except Exception:
        pass
    return None


async def stress(engine, requests: int, max_tokens: int, vocab: int, seed: int = 0, strict: bool = True,
                 tolerate: int = 0, prompt_range=(4, 96)) -> dict:
    rng = random.Random(seed)
    prompts = [[rng.randrange(vocab) for _ in range(rng.randint(*prompt_range))] for _ in range(max(1, requests // 2))]
    jobs = [p for p in prompts for _ in range(2)]
    rng.shuffle(jobs)
    res = await asyncio.gather(*(_run_one(engine, p, max_tokens) for p in jobs), return_exceptions=True)
    errors = [repr(r) for r in res if isinstance(r, BaseException)]
    ok = [r for r in res if not isinstance(r, BaseException)]
    bad_len = sum(1 for r in ok if len(r["tokens"]) != max_tokens)
    bad_tok = sum(1 for r in ok if any(not 0 <= t < vocab for t in r["tokens"]))
    by_prompt: dict[tuple, list[list[int]]] = {}
    for p, r in zip(jobs, res):
        if not isinstance(r, BaseException):
            by_prompt.setdefault(tuple(p), []).append(r["tokens"])
    mismatched = sum(1 for outs in by_prompt.values() if len(outs) == 2 and outs[0] != outs[1])
    passed = not errors and bad_len == 0 and bad_tok == 0 and (mismatched == 0 if strict else mismatched <= tolerate)
    return {"gate": "stress", "pass": passed, "requests": len(jobs), "errors": errors[:5], "wrong_length": bad_len,
            "out_of_vocab": bad_tok, "mismatched_pairs": mismatched, "pairs": len(by_prompt)}


async def soak(engine, seconds: float, concurrency: int, vocab: int, seed: int = 0, prompt_range=(8, 2048),
               output_range=(1, 256)) -> dict:
    rng = random.Random(seed)
    llm = engine.llm
    kv0, mem0 = _kv_free(llm), _device_bytes()
    t_end = time.perf_counter() + seconds
    done, errors, wrong, tokens = 0, [], 0, 0
    ttft, itl = [], []

    async def worker(wid: int):
        nonlocal done, wrong, tokens
        r2 = random.Random(seed * 1000 + wid)
        while time.perf_counter() < t_end:
            n_out = r2.randint(*output_range)
            prompt = [r2.randrange(vocab) for _ in range(r2.randint(*prompt_range))]
            try:
                r = await _run_one(engine, prompt, n_out)
            except Exception as e:  # noqa: BLE001 -- every failure is a gate finding
                errors.append(repr(e))
                continue
            done += 1
            tokens += len(r["tokens"])
            wrong += len(r["tokens"]) != n_out
            if r["ttft_s"] is not None:
                ttft.append(r["ttft_s"])
            itl.extend(r["itl_s"])

    t0 = time.perf_counter()
    await asyncio.gather(*(worker(i) for i in range(concurrency)))
    wall = time.perf_counter() - t0
    # drain: the engine must have nothing left
    for _ in range(200):
        if not llm.has_unfinished():
            break
        await asyncio.sleep(0.01)
    drained = not llm.has_unfinished()
    kv1, mem1 = _kv_free(llm), _device_bytes()
    kv_ok = kv0 is None or kv1 == kv0
    mem_ok = mem0 is None or mem1 <= mem0
    passed = not errors and wrong == 0 and drained and kv_ok and mem_ok and done > 0
    return {"gate": "soak", "pass": passed, "seconds": round(wall, 1), "requests": done, "errors": errors[:5],
            "wrong_length": wrong, "drained": drained, "kv_free_start": kv0, "kv_free_end": kv1,
            "device_bytes_start": mem0, "device_bytes_end": mem1, "tok_s": round(tokens / max(wall, 1e-9), 1),
            "ttft_p50_s": _pct(ttft, 50), "ttft_p99_s": _pct(ttft, 99), "itl_p50_s": _pct(itl, 50),
            "itl_p99_s": _pct(itl, 99)}


async def ttft_by_length(engine, lengths: list[int], vocab: int, reps: int = 3, max_tokens: int = 8,
                         seed: int = 0) -> dict:
    rng = random.Random(seed)
    rows = {}
    for n in lengths:
        ts, il = [], []
        for _ in range(reps):
            r = await _run_one(engine, [rng.randrange(vocab) for _ in range(n)], max_tokens)
            ts.append(r["ttft_s"])
            il.extend(r["itl_s"])
        rows[n] = {"ttft_median_s": statistics.median(ts), "itl_p50_s": _pct(il, 50), "itl_p99_s": _pct(il, 99)}
    return {"gate": "ttft", "pass": True, "by_prompt_tokens": rows}


def _build(args):
    from ..engine.llm import LLM
    from ..models.config import EngineConfig, model_config
    from .async_engine import AsyncEngine

    cfg = model_config(args.model)
    ec = EngineConfig(max_batch=args.max_batch, max_model_len=args.max_model_len,
                      max_prefill_tokens=args.max_prefill_tokens)
    eng = AsyncEngine(LLM(cfg, ec, seed=args.seed))
    eng.start()
    return eng, cfg.vocab


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("gate", choices=["stress", "soak", "ttft"])
    ap.add_argument("--model", default="tiny-hybrid")
    ap.add_argument("--max-batch", type=int, default=16)
    ap.add_argument("--max-model-len", type=int, default=16384)
    ap.add_argument("--max-prefill-tokens", type=int, default=8192)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--requests", type=int, default=48)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--seconds", type=float, default=900.0)
    ap.add_argument("--concurrency", type=int, default=24)
    ap.add_argument("--lengths", default="128,1024,8192")
    ap.add_argument("--lenient", action="store_true", help="stress: tolerate --tolerate mismatched duplicate pairs")
    ap.add_argument("--tolerate", type=int, default=0)
    a = ap.parse_args(argv)
    eng, vocab = _build(a)
    try:
        if a.gate == "stress":
            res = asyncio.run(stress(eng, a.requests, a.max_tokens, vocab, a.seed, strict=not a.lenient,
                                     tolerate=a.tolerate))
        elif a.gate == "soak":
            res = asyncio.run(soak(eng, a.seconds, a.concurrency, vocab, a.seed))
        else:
            res = asyncio.run(ttft_by_length(eng, [int(x) for x in a.lengths.split(",")], vocab))
    finally:
        eng.stop()
    print(json.dumps(res))
    return 0 if res["pass"] else 1


if __name__ == "__main__":
    sys.exit(main())
