"""Asyncio front for the synchronous engine.

The engine (an ``LLM``) runs on one dedicated thread, which owns every CUDA call. Requests arrive on
the event loop, cross to the engine thread through a lock-protected inbox, and the tokens of each
step flow back to per-request asyncio queues with ``call_soon_threadsafe``. With tensor parallelism
the same loop runs on every rank: rank 0 owns the inbox and broadcasts each step's admissions and
aborts to the other ranks over a CPU (gloo) group, so every rank's scheduler sees the same requests
in the same order and takes the same steps.
"""
from __future__ import annotations

import asyncio
import threading
import time
from dataclasses import dataclass, field

from ..engine.scheduler import SamplingParams


@dataclass
class RequestOutput:
    request_id: str
    new_tokens: list[int]
    finished: bool
    prompt_tokens: int = 0
    finish_reason: str | None = None


@dataclass
class _Req:
    rid: str
    prompt: list[int]
    params: SamplingParams
    loop: asyncio.AbstractEventLoop | None
    queue: asyncio.Queue | None
    seq: object = None
    emitted: int = 0
    t_arrive: float = field(default_factory=time.time)


class EngineMetrics:
    def __init__(self):
        self.requests = 0
        self.finished = 0
        self.prompt_tokens = 0
        self.generation_tokens = 0
        self.steps = 0
        self.step_time_s = 0.0
        self.ttft: list[float] = []
        self.errors = 0  # engine steps that raised (their requests ended with reason "error")
        self.last_error: str | None = None


class AsyncEngine:
    def __init__(self, llm, group=None, rank: int = 0, world: int = 1, idle_sleep: float = 0.001):
        self.llm = llm
        self.group, self.rank, self.world = group, rank, world
        self._lock = threading.Lock()
        self._inbox: list[_Req] = []
        self._aborts: list[str] = []
        self._live: dict[str, _Req] = {}
        self._stop = False
        self._idle_sleep = idle_sleep
        self.metrics = EngineMetrics()
        self._thread: threading.Thread | None = None
        self._counter = 0

    # ------------------------------------------------------------------ event-loop side
    def start(self) -> None:
        self._thread = threading.Thread(target=self._run, name="r9k-engine", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=30)

    def new_request_id(self) -> str:
        with self._lock:
            self._counter += 1
            return f"req-{self._counter}"

    async def generate(self, prompt: list[int], params: SamplingParams, request_id: str | None = None):
        """Async iterator of RequestOutput (new tokens of each engine step)."""
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        req = _Req(request_id or self.new_request_id(), list(prompt), params, loop, q)
        with self._lock:
            self._inbox.append(req)
        try:
            while True:
                out: RequestOutput = await q.get()
                yield out
                if out.finished:
                    return
        except (asyncio.CancelledError, GeneratorExit):
            self.abort(req.rid)
            raise

    def abort(self, rid: str) -> None:
        with self._lock:
            self._aborts.append(rid)

    # ------------------------------------------------------------------ engine thread
    def _exchange(self):
        """Take this step's admissions / aborts (rank 0) and share them with every rank."""
        with self._lock:
            new, self._inbox = self._inbox, []
            aborts, self._aborts = self._aborts, []
            stop = self._stop
        if self.world > 1:
            import torch.distributed as dist

            msg = [[(r.rid, r.prompt, r.params) for r in new], aborts, stop] if self.rank == 0 else [None, None, None]
            dist.broadcast_object_list(msg, src=0, group=self.group)
            if self.rank != 0:
                new = [_Req(rid, p, sp, None, None) for rid, p, sp in msg[0]]
                aborts, stop = msg[1], msg[2]
        return new, aborts, stop

    def _emit(self, req: _Req, toks: list[int], finished: bool, reason: str | None) -> None:
        if req.queue is None:
            return
        out = RequestOutput(req.rid, toks, finished, len(req.prompt), reason)
        req.loop.call_soon_threadsafe(req.queue.put_nowait, out)

    def _run(self) -> None:
        llm, m = self.llm, self.metrics
        while True:
            new, aborts, stop = self._exchange()
            if stop:
                return
            for r in new:
                r.seq = llm.add_request(r.prompt, r.params)
                self._live[r.rid] = r
                m.requests += 1
                m.prompt_tokens += len(r.prompt)
            for rid in aborts:
                r = self._live.pop(rid, None)
                if r is not None:
                    llm.abort(r.seq)
            if not llm.has_unfinished():
                time.sleep(self._idle_sleep)
                continue
            t0 = time.time()
            try:
                llm.step()
            except Exception as e:  # noqa: BLE001 -- a failed step must not strand the clients
                # every live request ends with reason "error"; the engine keeps serving new ones
                m.errors += 1
                m.last_error = repr(e)
                for rid in list(self._live):
                    r = self._live.pop(rid)
                    try:
                        llm.abort(r.seq)
                    except Exception:  # noqa: BLE001
                        pass
                    self._emit(r, [], True, "error")
                continue
            m.steps += 1
            m.step_time_s += time.time() - t0
            for rid in list(self._live):
                r = self._live[rid]
                s = r.seq
                if len(s.output) > r.emitted:
                    toks = s.output[r.emitted:]
                    if r.emitted == 0:
                        m.ttft.append(time.time() - r.t_arrive)
                    r.emitted = len(s.output)
                    m.generation_tokens += len(toks)
                    reason = None
                    if s.finished:
                        reason = "stop" if (s.output and s.output[-1] == s.params.eos_token_id) else "length"
                    self._emit(r, toks, s.finished, reason)
                elif s.finished:
                    self._emit(r, [], True, "length")
                if s.finished:
                    m.finished += 1
                    del self._live[rid]
