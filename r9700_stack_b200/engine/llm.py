"""Public serving API.

    llm = LLM(tiny_hybrid(), EngineConfig(max_batch=4))
    outs = llm.generate([[1, 2, 3]], SamplingParams(max_tokens=8))

``LLM`` owns the model (one tensor-parallel rank per process), the paged KV cache and recurrent-state
pools, the scheduler and the model runner. ``add_request`` / ``step`` expose the engine loop for
benchmarks and servers; ``generate`` runs it to completion.
"""
from __future__ import annotations

import math

import torch

from ..models.config import EngineConfig, HybridConfig, ParallelConfig
from .runner import ModelRunner
from .scheduler import SamplingParams, Scheduler, Sequence


class LLM:
    def __init__(self, model_cfg, engine_cfg: EngineConfig | None = None, par: ParallelConfig | None = None,
                 device=None, seed: int = 0, comm=None, model=None, drafter=None):
        self.engine_cfg = ec = engine_cfg or EngineConfig()
        self.par = par or ParallelConfig()
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if model is None:
            placement = None
            if ec.ep_placement:
                from ..parallel.ep_placement import load as load_placement

                placement = load_placement(ec.ep_placement)
            model = build_model(model_cfg, self.par, self.device, seed=seed, comm=comm, max_ctx=ec.max_model_len,
                                placement=placement)
        self.model = model
        blocks_per_seq = math.ceil(ec.max_model_len / ec.kv_block)
        num_blocks = ec.num_kv_blocks or (ec.max_batch * blocks_per_seq + 1)
        num_slots = ec.max_batch + 1
        model.alloc_caches(num_blocks, num_slots, ec.kv_block)
        self.scheduler = Scheduler(num_blocks, num_slots, ec.kv_block, ec.max_batch, ec.max_prefill_tokens,
                                   ec.max_model_len)
        max_tokens = max(ec.max_prefill_tokens, ec.max_batch * (1 + ec.spec_tokens))
        self.runner = ModelRunner(model, ec, ec.kv_block, max_tokens, ec.max_batch, blocks_per_seq)
        self.drafter = None
        self.spec_stats = {"steps": 0, "drafted": 0, "accepted": 0}
        if ec.spec_tokens > 0:
            model.alloc_spec(self.runner.ws, ec.max_batch * (1 + ec.spec_tokens))
            self.drafter = drafter if drafter is not None else make_drafter(
                ec.spec_method, model, ec, num_blocks, num_slots, seed)
        if ec.cuda_graphs:
            self.runner.capture_decode_graphs()

    # ------------------------------------------------------------------------------------------
    def add_request(self, prompt: list[int], params: SamplingParams | None = None) -> Sequence:
        seq = Sequence(list(prompt), params or SamplingParams())
        self.scheduler.add(seq)
        return seq

    def step(self) -> list[Sequence]:
        """One engine step (a prefill chunk or a decode step). Returns sequences that finished."""
        k = self.engine_cfg.spec_tokens if self.drafter is not None else 0
        out = self.scheduler.schedule(lookahead=1 + k)
        if out.kind == "idle":
            return []
        if out.kind == "decode" and self.drafter is not None:
            # speculative verification is greedy; requests that sample with temperature get no drafts
            drafts = self.drafter.drafts([c.seq for c in out.chunks if c.seq.params.temperature <= 0])
            toks, accepted = self.runner.execute_spec(out, drafts)
            st = self.spec_stats
            st["steps"] += 1
            st["drafted"] += sum(len(d) for d in drafts.values())
            st["accepted"] += sum(a - 1 for a in accepted.values())
            done = self.scheduler.finish_step(out, toks)
            self.drafter.after_step(self, out, accepted, drafts)
        else:
            toks = self.runner.execute(out)
            done = self.scheduler.finish_step(out, toks)
            if self.drafter is not None:
                self.drafter.after_step(self, out, None, None)
        if self.drafter is not None:
            for s in done:
                self.drafter.release(s)
        return done

    def abort(self, seq: Sequence) -> None:
        self.scheduler.abort(seq)
        if self.drafter is not None:
            self.drafter.release(seq)

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work

    def generate(self, prompts: list[list[int]], params: SamplingParams | None = None) -> list[list[int]]:
        seqs = [self.add_request(p, params) for p in prompts]
        while self.has_unfinished():
            self.step()
        return [s.output for s in seqs]


def make_drafter(method: str, model, ec: EngineConfig, num_blocks: int, num_slots: int, seed: int = 0):
    """The drafter named by ``EngineConfig.spec_method``: ngram | mtp | block | dspark."""
    from ..spec.drafters import DSparkDrafter, ModelDrafter, NgramDrafter

    if method == "ngram":
        return NgramDrafter(ec.spec_tokens)
    if method == "dspark":
        return DSparkDrafter(model, ec.spec_tokens, ec, num_blocks, num_slots, seed=seed)
    if method in ("mtp", "block"):
        return ModelDrafter(model, method, ec.spec_tokens, ec, num_blocks, num_slots, seed=seed)
    raise ValueError(f"unknown speculative method {method!r}")


def build_model(cfg, par, device, seed=0, comm=None, max_ctx: int = 32768, placement=None):
    if isinstance(cfg, HybridConfig):
        if cfg.moe_experts:
            from ..models.hybrid_moe import HybridMoELM

            return HybridMoELM(cfg, par, device, seed=seed, comm=comm, placement=placement)
        from ..models.hybrid import HybridLM

        return HybridLM(cfg, par, device, seed=seed, comm=comm)
    from ..models.dsv4 import DSV4Config, DSV4LM
    from ..models.mla_moe import MLAConfig, MLAMoELM

    if isinstance(cfg, DSV4Config):
        return DSV4LM(cfg, par, device, seed=seed, comm=comm, max_ctx=max_ctx)
    if isinstance(cfg, MLAConfig):
        return MLAMoELM(cfg, par, device, seed=seed, comm=comm, max_ctx=max_ctx)
    raise TypeError(f"unsupported model config {type(cfg)}")
