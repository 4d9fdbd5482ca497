"""OpenAI-compatible HTTP server over :class:`AsyncEngine`.

Endpoints: ``POST /v1/completions``, ``POST /v1/chat/completions`` (both with ``stream``), ``GET
/v1/models``, ``GET /health``, ``GET /metrics`` (Prometheus text: request, token, step and TTFT
counters, speculative acceptance). Prompts may be text (tokenised by the server's tokenizer) or
token-id lists. This is the API surface the reference exposes through ``vllm serve``
(serve/serve.sh:41-117); the benchmark clients of ``bench/harness.py`` and ours speak it.
"""
from __future__ import annotations

import json
import time
import uuid

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..engine.scheduler import SamplingParams


def _params(body: dict, tok) -> SamplingParams:
    mt = body.get("max_tokens", body.get("max_completion_tokens", 16))
    if not isinstance(mt, int) or mt < 1:
        raise HTTPException(400, "max_tokens must be a positive integer")
    ignore_eos = bool(body.get("ignore_eos", False))
    return SamplingParams(max_tokens=mt, temperature=float(body.get("temperature", 0.0) or 0.0),
                          top_k=int(body.get("top_k", 0) or 0), top_p=float(body.get("top_p", 1.0) or 1.0),
                          ignore_eos=ignore_eos, eos_token_id=tok.eos_token_id, seed=int(body.get("seed", 0) or 0))


def build_app(engine, tokenizer, model_name: str, max_model_len: int) -> FastAPI:
    app = FastAPI(title="r9700_stack_b200")

    def _prompt_ids(p) -> list[int]:
        if isinstance(p, list) and all(isinstance(x, int) for x in p):
            ids = list(p)
        elif isinstance(p, str):
            ids = tokenizer.encode(p)
        else:
            raise HTTPException(400, "prompt must be a string or a list of token ids")
        if not ids:
            raise HTTPException(400, "empty prompt")
        if any(not 0 <= x < tokenizer.vocab_size for x in ids):
            raise HTTPException(400, "token id out of range")
        return ids

    async def _run(ids, params, chat: bool, stream: bool):
        rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:16]
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        if len(ids) + params.max_tokens > max_model_len:
            raise HTTPException(400, f"prompt + max_tokens exceeds max_model_len ({max_model_len})")

        def choice(text, toks, reason, delta: bool):
            if chat:
                c = {"index": 0, "finish_reason": reason}
                c["delta" if delta else "message"] = {"role": "assistant", "content": text}
                return c
            return {"index": 0, "text": text, "token_ids": toks, "finish_reason": reason}

        if stream:
            async def gen():
                n = 0
                async for out in engine.generate(ids, params):
                    n += len(out.new_tokens)
                    chunk = {"id": rid, "object": obj + (".chunk" if chat else ""), "created": created,
                             "model": model_name,
                             "choices": [choice(tokenizer.decode(out.new_tokens), out.new_tokens,
                                                out.finish_reason, True)]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                usage = {"prompt_tokens": len(ids), "completion_tokens": n, "total_tokens": len(ids) + n}
                yield f"data: {json.dumps({'id': rid, 'object': obj, 'usage': usage, 'choices': []})}\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        toks, reason = [], None
        async for out in engine.generate(ids, params):
            toks += out.new_tokens
            reason = out.finish_reason
        body = {"id": rid, "object": obj, "created": created, "model": model_name,
                "choices": [choice(tokenizer.decode(toks), toks, reason, False)],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                          "total_tokens": len(ids) + len(toks)}}
        return JSONResponse(body)

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "r9700_stack_b200",
                                            "max_model_len": max_model_len}]}

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        p = body.get("prompt")
        if isinstance(p, list) and p and isinstance(p[0], (list, str)):
            if len(p) != 1:
                raise HTTPException(400, "one prompt per request")
            p = p[0]
        return await _run(_prompt_ids(p), _params(body, tokenizer), False, bool(body.get("stream", False)))

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            raise HTTPException(400, "messages must be a non-empty list")
        ids = _prompt_ids(tokenizer.apply_chat_template(msgs))
        return await _run(ids, _params(body, tokenizer), True, bool(body.get("stream", False)))

    @app.get("/metrics")
    async def metrics():
        m = engine.metrics
        lines = [
            f"r9k_requests_total {m.requests}",
            f"r9k_requests_finished_total {m.finished}",
            f"r9k_prompt_tokens_total {m.prompt_tokens}",
            f"r9k_generation_tokens_total {m.generation_tokens}",
            f"r9k_engine_steps_total {m.steps}",
            f"r9k_engine_step_seconds_total {m.step_time_s:.6f}",
        ]
        if m.ttft:
            srt = sorted(m.ttft)
            lines.append(f"r9k_ttft_seconds_p50 {srt[len(srt) // 2]:.6f}")
        st = getattr(engine.llm, "spec_stats", None)
        if st:
            lines += [f"r9k_spec_drafted_tokens_total {st['drafted']}",
                      f"r9k_spec_accepted_tokens_total {st['accepted']}",
                      f"r9k_spec_verify_steps_total {st['steps']}"]
        return PlainTextResponse("\n".join(lines) + "\n")

    return app
