"""Server launcher (the role of the reference's serve/serve.sh + per-model launchers).

    python -m r9700_stack_b200.serve.launch --model dense27b --port 8000
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m r9700_stack_b200.serve.launch --model dense27b
    python -m r9700_stack_b200.serve.launch --model flashnext --spec mtp --spec-tokens 3 --dry-run

One process per GPU. Rank 0 serves HTTP; every rank runs the engine loop, with rank 0 broadcasting
each step's admissions so all ranks schedule identically. Decode all-reduces use the fused NVLink
path (``SymmComm``); prefill-size messages use NCCL. ``--dry-run`` prints the resolved configuration
and the per-rank memory plan without touching a GPU.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="dense27b")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-batch", type=int, default=16)
    ap.add_argument("--max-model-len", type=int, default=32768)
    ap.add_argument("--max-prefill-tokens", type=int, default=8192)
    ap.add_argument("--kv-blocks", type=int, default=0, help="0: sized from max-batch x max-model-len")
    ap.add_argument("--spec", default="none", choices=["none", "ngram", "mtp", "block", "dspark"])
    ap.add_argument("--ep-placement", default="", help="JSON expert placement (parallel.ep_placement) for MoE models")
    ap.add_argument("--spec-tokens", type=int, default=0)
    ap.add_argument("--graph-sizes", default="1,2,4,8,16")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--tokenizer", default="", help="local Hugging Face tokenizer directory (default: bytes)")
    ap.add_argument("--served-model-name", default="")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--dry-run", action="store_true")
    return ap.parse_args(argv)


def plan(a) -> dict:
    from ..models.config import EngineConfig, model_config

    cfg = model_config(a.model)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    k = a.spec_tokens if a.spec != "none" else 0
    if a.spec != "none" and k == 0:
        k = cfg.draft_block - 1 if a.spec in ("block", "dspark") else 3
    ec = EngineConfig(max_batch=a.max_batch, max_model_len=a.max_model_len, max_prefill_tokens=a.max_prefill_tokens,
                      num_kv_blocks=a.kv_blocks, cuda_graphs=not a.no_graphs,
                      graph_batch_sizes=[int(x) for x in a.graph_sizes.split(",") if x],
                      spec_tokens=k, spec_method=a.spec if a.spec != "none" else "ngram", ep_placement=a.ep_placement)
    blocks = ec.num_kv_blocks or (ec.max_batch * math.ceil(ec.max_model_len / ec.kv_block) + 1)
    if hasattr(cfg, "attn_layers"):  # hybrid GDN / attention
        hkv = max(1, cfg.n_kv_heads // world)
        kv_bytes = len(cfg.attn_layers) * 2 * blocks * hkv * ec.kv_block * cfg.head_dim
        hv = cfg.gdn_v_heads // world
        state_b = 2 if cfg.gdn_state_dtype == "bf16" else 4
        ssm_bytes = len(cfg.gdn_layers) * (ec.max_batch + 1) * hv * cfg.gdn_head_dim ** 2 * state_b
    else:  # latent (MLA) cache: bf16 [512 | 64] rows + e4m3 indexer keys, replicated per rank
        kv_bytes = cfg.layers * blocks * ec.kv_block * (576 * 2 + 128)
        ssm_bytes = 0
    return {"model": cfg.name, "tp": world, "engine": ec.__dict__, "kv_blocks": blocks,
            "kv_cache_gb_per_rank": round(kv_bytes / 1e9, 2), "gdn_state_gb_per_rank": round(ssm_bytes / 1e9, 2),
            "cfg": cfg, "ec": ec}


def main(argv=None) -> int:
    a = parse(argv)
    p = plan(a)
    if a.dry_run:
        print(json.dumps({k: v for k, v in p.items() if k not in ("cfg", "ec")}, default=str, indent=1))
        return 0
    import torch
    import torch.distributed as dist

    from ..engine.llm import LLM
    from ..models.config import ParallelConfig
    from ..parallel.comm import init_distributed
    from .async_engine import AsyncEngine
    from .tokenizer import ByteTokenizer, HFTokenizer

    rank, world, local = init_distributed()
    dev = torch.device("cuda", local)
    cfg, ec = p["cfg"], p["ec"]
    comm, group = None, None
    if world > 1:
        from ..parallel.symm import SymmComm

        comm = SymmComm(cfg.hidden, max_tokens=ec.max_batch, calls_per_step=2 * cfg.layers, device=dev)
        group = dist.new_group(backend="gloo")
    llm = LLM(cfg, ec, ParallelConfig(tp_size=world, tp_rank=rank), device=dev, seed=a.seed, comm=comm)
    eng = AsyncEngine(llm, group=group, rank=rank, world=world)
    if rank != 0:
        eng._run()  # follows rank 0 until it broadcasts stop
        return 0
    import uvicorn

    from .openai_server import build_app

    tok = HFTokenizer(a.tokenizer) if a.tokenizer else ByteTokenizer(cfg.vocab)
    app = build_app(eng, tok, a.served_model_name or cfg.name, ec.max_model_len)
    eng.start()
    try:
        uvicorn.run(app, host=a.host, port=a.port, log_level="warning")
    finally:
        eng.stop()
    return 0


if __name__ == "__main__":
    sys.exit(main())
