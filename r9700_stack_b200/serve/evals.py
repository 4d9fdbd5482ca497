"""Accuracy gates: paired evaluation with McNemar's test, long-context needles, and the drafter
self-test. They run in process over ``LLM`` (or any object with ``generate(prompts, params)``).

    python -m r9700_stack_b200.serve.evals paired --model tiny-hybrid --tasks arith --n 200
    python -m r9700_stack_b200.serve.evals paired --tasks gsm8k.jsonl --tokenizer <dir> ...
    python -m r9700_stack_b200.serve.evals needles --model tiny-hybrid --ctx 4096 --depths 0.1,0.5,0.9
    python -m r9700_stack_b200.serve.evals drafter --model tiny-hybrid --spec block

* paired: the same items through a candidate and a baseline configuration (e.g. a new kernel vs
  ``R9K_*=stock``, TP=2 vs TP=1). Per item, correct or not; the discordant pairs (b: baseline right,
  candidate wrong; c: the opposite) decide McNemar's exact two-sided test (binomial, p = 0.5 over
  b + c). ``selftest`` runs one configuration twice, which measures the stack's own run-to-run
  disagreement before any comparison is trusted (reference: bench/eval.py:1-235 paired GSM8K +
  McNemar and its selftest).
  Tasks: a JSONL file of ``{"question": ..., "answer": ...}`` records (GSM8K's format, the final
  number after "####" is the answer), scored by the last number in the output; or the built-in
  ``arith`` task (generated integer sums, offline).
* needles: a key -> value line hidden at several depths of a long filler context; passes when the
  greedy continuation after the query reproduces the value (reference: bench/ds41/needle.py).
* drafter: greedy generation with speculative decoding must equal generation without it token for
  token, since verification only accepts the target's own argmax (reference:
  bench/ds41/drafter_selftest.py -- the post-launch check that caught a silent drafter bug).
"""
from __future__ import annotations

import argparse
import json
import math
import random
import re
import sys

from ..engine.scheduler import SamplingParams
from .tokenizer import ByteTokenizer, HFTokenizer

_NUM = re.compile(r"-?\d+(?:\.\d+)?")


# ------------------------------------------------------------------------------------------------
# statistics
# ------------------------------------------------------------------------------------------------
def mcnemar_exact(b: int, c: int) -> float:
    """Two-sided exact McNemar p-value for b and c discordant pairs (binomial with p = 1/2)."""
    n = b + c
    if n == 0:
        return 1.0
    k = min(b, c)
    tail = sum(math.comb(n, i) for i in range(k + 1)) / 2.0 ** n
    return min(1.0, 2.0 * tail)


def paired_summary(base: list[bool], cand: list[bool], alpha: float = 0.05) -> dict:
    assert len(base) == len(cand)
    b = sum(1 for x, y in zip(base, cand) if x and not y)
    c = sum(1 for x, y in zip(base, cand) if y and not x)
    p = mcnemar_exact(b, c)
    n = len(base)
    return {"n": n, "baseline_correct": sum(base), "candidate_correct": sum(cand), "b_base_only": b,
            "c_cand_only": c, "p_value": p, "different": p < alpha,
            "pass": not (p < alpha and c < b)}  # fail only on a significant loss


# ------------------------------------------------------------------------------------------------
# tasks
# ------------------------------------------------------------------------------------------------
def arith_task(n: int, seed: int = 0) -> list[dict]:
    """Generated integer sums (offline stand-in with GSM8K's record format)."""
    rng = random.Random(seed)
    items = []
    for _ in range(n):
        a, b = rng.randint(10, 999), rng.randint(10, 999)
        items.append({"question": f"What is {a} + {b}?", "answer": f"{a} + {b} = {a + b} #### {a + b}"})
    return items


def load_jsonl(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def reference_answer(item: dict) -> str:
    ans = str(item["answer"])
    return ans.split("####")[-1].strip().replace(",", "")


def extract_answer(text: str) -> str | None:
    nums = _NUM.findall(text.replace(",", ""))
    return nums[-1] if nums else None


def score(text: str, item: dict) -> bool:
    got = extract_answer(text)
    if got is None:
        return False
    try:
        return abs(float(got) - float(reference_answer(item))) < 1e-6
    except ValueError:
        return got == reference_answer(item)


def run_items(llm, tok, items: list[dict], max_tokens: int = 64, batch: int = 16) -> list[tuple[str, bool]]:
    out = []
    params = SamplingParams(max_tokens=max_tokens, temperature=0.0)
    for i in range(0, len(items), batch):
        chunk = items[i:i + batch]
        prompts = [tok.encode(f"Question: {it['question']}\nAnswer:") for it in chunk]
        gens = llm.generate(prompts, params)
        for it, g in zip(chunk, gens):
            text = tok.decode(g)
            out.append((text, score(text, it)))
    return out


def paired(base_llm, cand_llm, tok, items, max_tokens: int = 64, alpha: float = 0.05) -> dict:
    base = [ok for _, ok in run_items(base_llm, tok, items, max_tokens)]
    cand = [ok for _, ok in run_items(cand_llm, tok, items, max_tokens)]
    return paired_summary(base, cand, alpha)


def selftest(llm, tok, items, max_tokens: int = 64) -> dict:
    """The same configuration twice: text disagreement rate and McNemar over the two runs."""
    r1 = run_items(llm, tok, items, max_tokens)
    r2 = run_items(llm, tok, items, max_tokens)
    s = paired_summary([ok for _, ok in r1], [ok for _, ok in r2])
    s["text_disagreement"] = sum(1 for (a, _), (b, _) in zip(r1, r2) if a != b) / max(1, len(items))
    s["pass"] = s["text_disagreement"] == 0.0 or not s["different"]
    return s


# ------------------------------------------------------------------------------------------------
# needles and drafter
# ------------------------------------------------------------------------------------------------
def needle_prompt(ctx_tokens: int, depth: float, key: list[int], value: list[int], vocab: int,
                  seed: int = 0) -> list[int]:
    """Filler ids with ``key + value`` inserted at ``depth`` (0..1) of the context, then ``key`` again
    as the query; the expected continuation is ``value``."""
    rng = random.Random(seed)
    n_fill = max(0, ctx_tokens - 2 * len(key) - len(value))
    fill = [rng.randrange(8, vocab) for _ in range(n_fill)]
    at = int(depth * n_fill)
    return fill[:at] + key + value + fill[at:] + key


def needles(llm, ctx_tokens: int, depths: list[float], vocab: int, trials: int = 1, seed: int = 0) -> dict:
    rng = random.Random(seed)
    hits, rows = 0, []
    for d in depths:
        for t in range(trials):
            key = [rng.randrange(8, vocab) for _ in range(4)]
            value = [rng.randrange(8, vocab) for _ in range(4)]
            prompt = needle_prompt(ctx_tokens, d, key, value, vocab, seed=seed + t)
            got = llm.generate([prompt], SamplingParams(max_tokens=len(value), temperature=0.0))[0]
            ok = got == value
            hits += ok
            rows.append({"depth": d, "trial": t, "ok": ok})
    n = len(depths) * trials
    return {"ctx": ctx_tokens, "found": hits, "n": n, "rows": rows, "pass": hits == n}


def drafter_selftest(plain_llm, spec_llm, prompts: list[list[int]], max_tokens: int = 32) -> dict:
    """Greedy tokens with and without speculative decoding must be identical."""
    params = SamplingParams(max_tokens=max_tokens, temperature=0.0)
    a = plain_llm.generate(prompts, params)
    b = spec_llm.generate(prompts, params)
    diff = [i for i, (x, y) in enumerate(zip(a, b)) if x != y]
    st = getattr(spec_llm, "spec_stats", {})
    acc = st.get("accepted", 0) / max(1, st.get("drafted", 0)) if st else None
    return {"prompts": len(prompts), "mismatched": diff, "acceptance": acc, "pass": not diff}


# ------------------------------------------------------------------------------------------------
# CLI
# ------------------------------------------------------------------------------------------------
def _llm(args, spec: str = ""):
    from ..engine.llm import LLM
    from ..models.config import EngineConfig, model_config

    cfg = model_config(args.model)
    ec = EngineConfig(max_batch=16, max_model_len=args.max_len, max_prefill_tokens=min(args.max_len, 8192))
    if spec:
        ec.spec_tokens, ec.spec_method = 4, spec
    return LLM(cfg, ec, seed=args.seed), cfg


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("paired", "selftest", "needles", "drafter"):
        p = sub.add_parser(name)
        p.add_argument("--model", default="tiny-hybrid")
        p.add_argument("--seed", type=int, default=0)
        p.add_argument("--max-len", type=int, default=8192)
        if name in ("paired", "selftest"):
            p.add_argument("--tasks", default="arith")
            p.add_argument("--n", type=int, default=100)
            p.add_argument("--max-tokens", type=int, default=64)
            p.add_argument("--tokenizer", default="")
        if name == "paired":
            p.add_argument("--candidate-env", default="", help="KEY=VAL,... knobs of the candidate run")
        if name == "needles":
            p.add_argument("--ctx", type=int, default=4096)
            p.add_argument("--depths", default="0.1,0.5,0.9")
        if name == "drafter":
            p.add_argument("--spec", default="ngram")
    a = ap.parse_args(argv)
    if a.cmd in ("paired", "selftest"):
        items = arith_task(a.n, a.seed) if a.tasks == "arith" else load_jsonl(a.tasks)[: a.n]
        tok = HFTokenizer(a.tokenizer) if a.tokenizer else ByteTokenizer()
        base, _ = _llm(a)
        if a.cmd == "selftest":
            res = selftest(base, tok, items, a.max_tokens)
        else:
            import os

            from .. import knobs

            for kv in filter(None, a.candidate_env.split(",")):
                k, v = kv.split("=", 1)
                os.environ[k] = v
            knobs.refresh()
            cand, _ = _llm(a)
            res = paired(base, cand, tok, items, a.max_tokens)
    elif a.cmd == "needles":
        llm, cfg = _llm(a)
        res = needles(llm, a.ctx, [float(x) for x in a.depths.split(",")], cfg.vocab)
    else:
        plain, cfg = _llm(a)
        spec, _ = _llm(a, spec=a.spec)
        rng = random.Random(a.seed)
        prompts = [[rng.randrange(8, cfg.vocab) for _ in range(rng.randrange(8, 64))] for _ in range(8)]
        res = drafter_selftest(plain, spec, prompts)
    print(json.dumps(res))
    return 0 if res.get("pass") else 1


if __name__ == "__main__":
    sys.exit(main())
