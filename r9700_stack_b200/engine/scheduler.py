"""Continuous-batching scheduler.

Each step is either a prefill step (chunks of waiting prompts, up to ``max_prefill_tokens``) or a
decode step (one token per running sequence, or 1 + k draft tokens under speculative decoding).
KV blocks are allocated as sequences grow; a sequence that cannot get a block is preempted back to
the waiting queue (recompute). This is the role stock vLLM's scheduler plays for the reference.
"""
from __future__ import annotations

import itertools
from collections import deque
from dataclasses import dataclass, field

from .cache import BlockAllocator, SlotAllocator


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    ignore_eos: bool = True
    eos_token_id: int = -1
    seed: int = 0


_ids = itertools.count()


@dataclass
class Sequence:
    prompt: list[int]
    params: SamplingParams
    seq_id: int = field(default_factory=lambda: next(_ids))
    output: list[int] = field(default_factory=list)
    num_computed: int = 0  # tokens whose KV/state is in the cache
    blocks: list[int] = field(default_factory=list)
    state_slot: int = -1
    finished: bool = False

    @property
    def tokens(self) -> list[int]:
        return self.prompt + self.output

    @property
    def length(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def prefill_done(self) -> bool:
        return self.num_computed >= len(self.prompt)


@dataclass
class ScheduledChunk:
    seq: Sequence
    start: int  # first token position processed in this step
    n: int  # tokens processed
    sample: bool  # whether a token is sampled from the last position


@dataclass
class SchedulerOutput:
    kind: str  # "prefill" | "decode" | "idle"
    chunks: list[ScheduledChunk]

    @property
    def num_tokens(self) -> int:
        return sum(c.n for c in self.chunks)


class Scheduler:
    def __init__(self, num_blocks: int, num_slots: int, block_size: int, max_batch: int,
                 max_prefill_tokens: int, max_model_len: int):
        self.blocks = BlockAllocator(num_blocks)
        self.slots = SlotAllocator(num_slots)
        self.block_size = block_size
        self.max_batch = max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.max_model_len = max_model_len
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []
        self.finished: list[Sequence] = []

    def add(self, seq: Sequence) -> None:
        if len(seq.prompt) + seq.params.max_tokens > self.max_model_len:
            raise ValueError("prompt + max_tokens exceeds max_model_len")
        self.waiting.append(seq)

    @property
    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def _blocks_needed(self, seq: Sequence, upto: int) -> int:
        need = (upto + self.block_size - 1) // self.block_size
        return max(0, need - len(seq.blocks))

    def _grow(self, seq: Sequence, upto: int) -> bool:
        n = self._blocks_needed(seq, upto)
        if n == 0:
            return True
        if not self.blocks.can_allocate(n):
            return False
        seq.blocks.extend(self.blocks.allocate(n))
        return True

    def ensure(self, seq: Sequence, upto: int) -> bool:
        """Make sure the blocks of ``seq`` cover positions < upto (drafters write ahead)."""
        if upto > self.max_model_len + 64:
            return False
        return self._grow(seq, upto)

    def _release(self, seq: Sequence) -> None:
        if seq.blocks:
            self.blocks.free(seq.blocks)
            seq.blocks = []
        if seq.state_slot >= 0:
            self.slots.free_one(seq.state_slot)
            seq.state_slot = -1

    def abort(self, seq: Sequence) -> None:
        """Drop a request wherever it is (waiting or running) and free its blocks and state slot."""
        if seq.finished:
            return
        if seq in self.waiting:
            self.waiting.remove(seq)
        if seq in self.running:
            self.running.remove(seq)
        self._release(seq)
        seq.finished = True
        self.finished.append(seq)

    def preempt(self, seq: Sequence) -> None:
        self._release(seq)
        seq.num_computed = 0
        seq.prompt = seq.prompt + seq.output
        seq.output = []
        self.running.remove(seq)
        self.waiting.appendleft(seq)

    def schedule(self, lookahead: int = 1) -> SchedulerOutput:
        # prefill first (prompt chunks), so new requests join the decode batch quickly
        chunks: list[ScheduledChunk] = []
        budget = self.max_prefill_tokens
        prefilling = [s for s in self.running if not s.prefill_done]
        candidates = prefilling + list(self.waiting)
        for seq in candidates:
            if budget <= 0:
                break
            if seq in self.waiting:
                if len(self.running) >= self.max_batch or self.slots.num_free == 0:
                    break
            n = min(len(seq.prompt) - seq.num_computed, budget)
            if not self._grow(seq, seq.num_computed + n):
                break
            if seq in self.waiting:
                self.waiting.remove(seq)
                seq.state_slot = self.slots.allocate_one()
                self.running.append(seq)
            last = seq.num_computed + n >= len(seq.prompt)
            chunks.append(ScheduledChunk(seq, seq.num_computed, n, sample=last))
            budget -= n
        if chunks:
            return SchedulerOutput("prefill", chunks)
        # decode: every running sequence advances by `lookahead` positions (1 + draft tokens)
        for seq in list(self.running):
            if not self._grow(seq, seq.length + lookahead):
                victim = self.running[-1]
                self.preempt(victim)
                if victim is seq:
                    continue
                if not self._grow(seq, seq.length + lookahead):
                    continue
        dec = [ScheduledChunk(s, s.length - 1, 1, sample=True) for s in self.running if s.prefill_done]
        return SchedulerOutput("decode" if dec else "idle", dec)

    def finish_step(self, out: SchedulerOutput, new_tokens: dict[int, list[int]]) -> list[Sequence]:
        done = []
        for ch in out.chunks:
            seq = ch.seq
            if out.kind == "prefill":
                seq.num_computed += ch.n
            toks = new_tokens.get(seq.seq_id, [])
            for t in toks:
                if len(seq.output) >= seq.params.max_tokens:
                    break
                seq.output.append(t)
                if not seq.params.ignore_eos and t == seq.params.eos_token_id:
                    break
            if out.kind == "decode":
                # every token but the newest is in the cache (a verify step commits the accepted drafts)
                seq.num_computed = seq.length - 1
            if len(seq.output) >= seq.params.max_tokens or (
                not seq.params.ignore_eos and seq.output and seq.output[-1] == seq.params.eos_token_id
            ):
                seq.finished = True
                self.running.remove(seq)
                self._release(seq)
                self.finished.append(seq)
                done.append(seq)
        return done
