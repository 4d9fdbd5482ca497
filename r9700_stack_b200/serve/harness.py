"""Benchmark client for a running server (the role of the reference's bench/harness.py and
bench/bench.py): concurrent streaming completions with nonce-prefixed prompts, TTFT, per-stream
decode rate and aggregate throughput, medians and coefficient of variation over repetitions.

    python -m r9700_stack_b200.serve.harness --url http://127.0.0.1:8000 --streams 1,8,16 \
        --prompt-tokens 8192 --max-tokens 512 --reps 3 --jsonl results.jsonl
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import statistics
import time


async def one_request(session, url: str, prompt: list[int], max_tokens: int) -> dict:
    body = {"prompt": prompt, "max_tokens": max_tokens, "stream": True, "ignore_eos": True, "temperature": 0}
    t0 = time.perf_counter()
    ttft, n, stamps = None, 0, []
    async with session.post(url + "/v1/completions", json=body) as r:
        if r.status != 200:
            raise RuntimeError(f"HTTP {r.status}: {await r.text()}")
        async for raw in r.content:
            line = raw.decode().strip()
            if not line.startswith("data:") or line == "data: [DONE]":
                continue
            d = json.loads(line[5:])
            for c in d.get("choices", []):
                k = len(c.get("token_ids") or [])
                if k:
                    now = time.perf_counter()
                    if ttft is None:
                        ttft = now - t0
                    n += k
                    stamps.append(now)
    t1 = time.perf_counter()
    dec = (n - 1) / (stamps[-1] - stamps[0]) if n > 1 and stamps[-1] > stamps[0] else None
    return {"ttft_s": ttft, "tokens": n, "total_s": t1 - t0, "decode_tok_s": dec}


async def run_level(url: str, streams: int, prompt_tokens: int, max_tokens: int, vocab: int, seed: int) -> dict:
    import aiohttp

    rng = random.Random(seed)
    prompts = []
    for i in range(streams):
        nonce = [rng.randrange(3, vocab) for _ in range(8)]  # defeats any prefix cache
        prompts.append(nonce + [rng.randrange(3, vocab) for _ in range(prompt_tokens - 8)])
    timeout = aiohttp.ClientTimeout(total=3600)
    async with aiohttp.ClientSession(timeout=timeout) as s:
        t0 = time.perf_counter()
        res = await asyncio.gather(*[one_request(s, url, p, max_tokens) for p in prompts])
        wall = time.perf_counter() - t0
    toks = sum(r["tokens"] for r in res)
    return {"streams": streams, "aggregate_tok_s": toks / wall, "wall_s": wall,
            "ttft_s_median": statistics.median(r["ttft_s"] for r in res),
            "decode_tok_s_median": statistics.median(r["decode_tok_s"] or 0.0 for r in res)}


def summarize(runs: list[dict]) -> dict:
    agg = [r["aggregate_tok_s"] for r in runs]
    med = statistics.median(agg)
    cv = statistics.pstdev(agg) / med if med and len(agg) > 1 else 0.0
    return {"streams": runs[0]["streams"], "aggregate_tok_s_median": med, "cv": cv,
            "ttft_s_median": statistics.median(r["ttft_s_median"] for r in runs),
            "decode_tok_s_median": statistics.median(r["decode_tok_s_median"] for r in runs), "reps": len(runs)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--streams", default="1,16")
    ap.add_argument("--prompt-tokens", type=int, default=512)
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--vocab", type=int, default=259)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--jsonl", default="")
    a = ap.parse_args(argv)
    out = []
    for n in [int(x) for x in a.streams.split(",")]:
        runs = [asyncio.run(run_level(a.url, n, a.prompt_tokens, a.max_tokens, a.vocab, seed=1000 * n + r))
                for r in range(a.reps)]
        s = summarize(runs)
        out.append(s)
        print(json.dumps(s), flush=True)
        if a.jsonl:
            with open(a.jsonl, "a") as f:
                for r in runs:
                    f.write(json.dumps(r) + "\n")
    return out


if __name__ == "__main__":
    main()
