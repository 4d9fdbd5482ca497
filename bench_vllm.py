"""Stock-vLLM comparison arm of bench.py (``--impl vllm``).

The same architecture as the headline benchmark: the Qwen3.5 dense hybrid layout of 64 layers, 3:1
Gated-DeltaNet to full attention, hidden 5120, ffn 17408, vocab 248320, GDN 16 key / 48 value heads
of 128, attention 24 q / 4 kv heads of 256. It is served by the image's unmodified vLLM with dummy
(random) bf16 weights: cuBLAS GEMMs, vLLM's own attention and GDN kernels, NCCL all-reduces, CUDA
graphs. None of this repository's kernels or engine is on this path. This is not the reference
(a ROCm/gfx1201 plugin that cannot run on CUDA); it is the second comparator, stock vLLM with
NCCL + cuBLAS on the same box.

Under torchrun every rank builds the engine with vLLM's ``external_launcher`` executor (one rank per
GPU, the same SPMD steps). Timing is wall clock around engine steps bracketed by
``torch.cuda.synchronize()`` and a barrier, max over ranks. vLLM schedules and launches from the host
inside each step, so this is an end-to-end figure.
"""
from __future__ import annotations

import json
import os
import tempfile
import time


def _config_dir(layers: int) -> str:
    import transformers

    text = dict(
        hidden_size=5120, intermediate_size=17408, num_hidden_layers=layers, vocab_size=248320,
        num_attention_heads=24, num_key_value_heads=4, head_dim=256, partial_rotary_factor=0.25,
        rope_theta=10000000.0, rms_norm_eps=1e-6, linear_conv_kernel_dim=4, linear_key_head_dim=128,
        linear_value_head_dim=128, linear_num_key_heads=16, linear_num_value_heads=48,
        layer_types=["full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(layers)],
        max_position_embeddings=32768, tie_word_embeddings=False,
    )
    cfg = transformers.Qwen3_5Config(text_config=text)
    cfg.architectures = ["Qwen3_5ForConditionalGeneration"]
    d = tempfile.mkdtemp(prefix="r9k_vllm_model_")
    cfg.save_pretrained(d)
    return d


def run(args, metric: str) -> int:
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # engine core in this process
    try:
        import numpy as np
        import torch
        from vllm import LLM, SamplingParams
        from vllm.inputs import TokensPrompt

        layers = args.layers or 64
        S, P = args.streams, args.prompt_len
        kw = dict(model=_config_dir(layers), load_format="dummy", dtype="bfloat16", tensor_parallel_size=world,
                  max_model_len=P + args.warmup + 2 * args.steps + 256, max_num_seqs=S, seed=0,
                  gpu_memory_utilization=0.85, skip_tokenizer_init=True, enable_prefix_caching=False,
                  limit_mm_per_prompt={"image": 0, "video": 0})
        if world > 1:
            kw["distributed_executor_backend"] = "external_launcher"
        t0 = time.time()
        llm = LLM(**kw)
        build_s = time.time() - t0
        eng = llm.llm_engine
        rng = np.random.default_rng(1234)
        prompt = lambda: TokensPrompt(prompt_token_ids=rng.integers(0, 248320, P).tolist())

        def sync():
            torch.cuda.synchronize()
            if world > 1 and torch.distributed.is_initialized():
                torch.distributed.barrier()
            torch.cuda.synchronize()

        def max_ranks(x: float) -> float:
            if world > 1 and torch.distributed.is_initialized():
                t = torch.tensor([x], dtype=torch.float64, device="cuda")
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                return float(t)
            return x

        # prefill @8k, one stream: one warm-up, two timed
        pre = []
        for it in range(3):
            sync()
            a = time.perf_counter()
            llm.generate([prompt()], SamplingParams(max_tokens=1, ignore_eos=True), use_tqdm=False)
            sync()
            if it:
                pre.append((time.perf_counter() - a) * 1e3)
        pre_ms = max_ranks(max(pre))

        # decode, S streams: prefill them, W warm-up steps, K timed steps (one token per stream each)
        total = args.warmup + args.steps + 8
        sp = SamplingParams(max_tokens=total, ignore_eos=True)
        for i in range(S):
            eng.add_request(f"d{i}", prompt(), sp)
        produced = {}
        while len(produced) < S or min(produced.values()) < 1:
            for o in eng.step():
                produced[o.request_id] = len(o.outputs[0].token_ids)
        for _ in range(args.warmup):
            eng.step()
        sync()
        a = time.perf_counter()
        for _ in range(args.steps):
            eng.step()
        sync()
        dec_ms = max_ranks((time.perf_counter() - a) * 1e3)
        while eng.has_unfinished_requests():
            eng.step()
        if rank == 0:
            v = S * args.steps / (dec_ms / 1e3)
            print(json.dumps({
                "impl": "vllm", "metric": metric, "value": round(v, 2), "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dec_ms / args.steps, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16 (stock)",
                "data": "synthetic: vLLM dummy (random) weights of the named architecture, uniform random prompt ids",
                "timing": "wall clock of engine steps, synchronize + barrier on both sides, max over ranks",
                "config": {"model": f"Qwen3_5ForConditionalGeneration text stack, {layers} layers (hybrid-dense-27b shape)",
                           "global_batch": S, "seq_len": P, "parallelism": f"tp{world}",
                           "collectives": "NCCL (vLLM stock)"},
                "decode_16_streams_tok_s": round(v, 2), "prefill_8k_tok_s": round(P / (pre_ms / 1e3), 1),
                "prefill_8k_ms": round(pre_ms, 2), "build_s": round(build_s, 1),
                "vllm": __import__("vllm").__version__,
            }), flush=True)
        return 0
    except Exception as e:  # noqa: BLE001 - report what stock vLLM did on this box
        if rank == 0:
            print(json.dumps({"impl": "vllm", "metric": metric,
                              "unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:300] if str(e) else ''}"}),
                  flush=True)
        return 0
