"""Kernel micro-benchmark: one kernel family at one shape, CUDA-event timed, with a roofline fraction.

    python -m r9700_stack_b200.tuning.kbench gemm --N 5120 --K 17408 --M 16 --fmt fp4
    python -m r9700_stack_b200.tuning.kbench gemm --N 17408 --K 5120 --M 16 --fmt fp4 --swiglu
    python -m r9700_stack_b200.tuning.kbench moe --T 16 --E 288 --topk 10 --H 2048 --I 512
    python -m r9700_stack_b200.tuning.kbench gemm ... --reps 1 --warmup 0     # one launch (for ncu -c 1)
    python -m r9700_stack_b200.tuning.kbench qsa --S 16 --ctx 8192 --topk 512     # QSA sparse decode attention
    python -m r9700_stack_b200.tuning.kbench hc --T 16 --hc 4 --H 2048             # fused hyper-connection point
    python -m r9700_stack_b200.tuning.kbench decode --model dense27b --streams 16 --reps 2 --eager
        # eager decode steps of a whole model inside NVTX ranges "decode_step" (ncu --nvtx-include)

Timed calls are captured into a CUDA graph and replayed (device time only) unless --eager.

Weights rotate over enough copies that one pass over them exceeds L2 (126 MB), so every timed launch
streams its weights from HBM; achieved bandwidth is algorithmic bytes / event time and the fraction is
taken against the measured copy bandwidth and bf16 GEMM rate in MEASURED_PEAKS.json at the repository
root (falling back to 6.65 TB/s and 1.59 PFLOP/s). The reference's counterparts are its graph-timed
sweeps (tuning/tune_dense.py, tuning/decode_moe_sweep.py).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
L2_BYTES = 126 * 2**20


def peaks() -> dict:
    p = os.path.join(HERE, "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "src": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def _time(fn, reps: int, warmup: int, graph: bool = True) -> float:
    """Device time per call (us). The timed calls are captured into one CUDA graph and replayed, so
    host launch overhead is excluded; ``graph=False`` times eager launches instead."""
    from ..utils import status

    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    if reps <= 0:
        return 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(reps):
                    fn(i)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()  # first replay uploads the graph
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
    else:
        e0.record()
        for i in range(reps):
            fn(i)
        e1.record()
    torch.cuda.synchronize()
    status.check()
    return e0.elapsed_time(e1) * 1e3 / reps  # us


def bench_gemm(a) -> dict:
    from ..ops import linear as L

    torch.manual_seed(0)
    N, K, M = a.N, a.K, a.M
    fp4 = a.fmt == "fp4"
    per = N * K * (2 if a.fmt == "bf16" else (0.5 if fp4 else 1.0)) * (2 if a.swiglu else 1)
    nw = max(1, min(a.max_copies, int(2 * L2_BYTES // per) + 1))

    def mk():
        w = torch.randn(N, K, device="cuda") * 0.02
        if a.fmt == "bf16":
            return L.BF16Weight(w.bfloat16())
        return L.mx_from_float(w, fp4=fp4, search=False, tiled=a.tiled)

    ws = [(mk(), mk()) if a.swiglu else mk() for _ in range(nw)]
    xb = torch.randn(M, K, device="cuda").bfloat16()
    if a.fmt == "bf16":
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        if a.swiglu:
            f = lambda i: L.bf16_swiglu(xb, ws[i % nw][0], ws[i % nw][1], out=out)
        else:
            f = lambda i: L.bf16_linear(xb, ws[i % nw], out=out)
    else:
        x = L.quant_act(xb)
        if a.swiglu:
            o = L.alloc_act(M, N, "cuda")
            f = lambda i: L.mx_swiglu(x, ws[i % nw][0], ws[i % nw][1], out=o)
        else:
            out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            f = lambda i: L.mx_linear(x, ws[i % nw], out=out)
    tr = None
    if getattr(a, "trace", False):
        tr = torch.zeros(12 << 16, dtype=torch.int64, device="cuda")
        torch.ops.r9k.gemm_trace(tr)
    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    if tr is not None:
        torch.ops.r9k.gemm_trace(None)
    wbytes = per + (N * K // 32) * (0 if a.fmt == "bf16" else 1) * (2 if a.swiglu else 1)
    flops = 2.0 * M * N * K * (2 if a.swiglu else 1)
    r = {"kernel": "gemm", "fmt": a.fmt, "swiglu": a.swiglu, "N": N, "K": K, "M": M, "copies": nw,
         "us": us, "weight_bytes": wbytes, "flops": flops}
    if tr is not None:
        r["trace"] = trace_summary(tr)
    if a.vs_torch and a.fmt == "bf16" and not a.swiglu:
        # the library baseline: torch.matmul (cuBLAS) on the same rotated bf16 weights, same timing
        tw = [w.w for w in ws]
        r["torch_matmul_us"] = _time(lambda i: torch.matmul(xb, tw[i % nw].T), a.reps, a.warmup, graph=not a.eager)
    return r


TRACE_POINTS = ("entry", "setup", "pdl", "first", "issued", "acc", "done", "done_t0", "parked", "sync1", "reduced",
                "sync2")


def trace_summary(buf: torch.Tensor) -> dict:
    """Per-phase timing of the last traced GEMM launch (gemm_trace stamps, 12 per CTA): each point's
    min / median / max over CTAs in us from the first CTA's entry, and the median of each phase."""
    t = buf.view(-1, 12)[:, : len(TRACE_POINTS)].cpu()
    t = t[t[:, 0] > 0]
    if t.numel() == 0:
        return {}
    rel = (t - t[:, 0].min()).double() / 1e3
    out = {"ctas": int(t.shape[0])}
    for i, name in enumerate(TRACE_POINTS):
        col = rel[:, i][t[:, i] > 0]
        if col.numel():
            out[name] = [round(float(col.min()), 2), round(float(col.median()), 2), round(float(col.max()), 2)]
    ph = {}
    for i in range(1, len(TRACE_POINTS)):
        ok = (t[:, i] > 0) & (t[:, i - 1] > 0)
        if ok.any():
            d = (t[ok, i] - t[ok, i - 1]).double() / 1e3
            ph[f"{TRACE_POINTS[i - 1]}->{TRACE_POINTS[i]}"] = round(float(d.median()), 2)
    for a, b in (("acc", "parked"), ("parked", "sync1"), ("sync1", "reduced"), ("reduced", "sync2"), ("sync2", "done")):
        ia, ib = TRACE_POINTS.index(a), TRACE_POINTS.index(b)
        ok = (t[:, ia] > 0) & (t[:, ib] > 0)
        if ok.any():
            ph[f"{a}->{b}"] = round(float(((t[ok, ib] - t[ok, ia]).double() / 1e3).median()), 2)
    out["phase_median_us"] = ph
    return out


def bench_moe(a) -> dict:
    from .. import _native
    from ..ops import linear as L
    from ..utils import status

    torch.manual_seed(0)
    T, E, k, H, I = a.T, a.E, a.topk, a.H, a.I
    ops = _native.ops()
    G = L.stack_experts([L.mx_from_float(torch.randn(I, H, device="cuda") * 0.02, search=False) for _ in range(E)])
    U = L.stack_experts([L.mx_from_float(torch.randn(I, H, device="cuda") * 0.02, search=False) for _ in range(E)])
    D = L.stack_experts([L.mx_from_float(torch.randn(H, I, device="cuda") * 0.02, search=False) for _ in range(E)])
    x = L.quant_act(torch.randn(T, H, device="cuda").bfloat16())
    logits = torch.randn(T, E, device="cuda")
    A = T * k
    per_expert = A / max(1, min(E, A))  # token tile as moe_ffn picks it
    BN = 16 if per_expert <= 16 else 32 if per_expert <= 32 else 64 if per_expert <= 64 else 128
    max_rows = A + 256 * min(E, A)
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    perm = torch.empty(A, dtype=torch.int32, device="cuda")
    seg = torch.empty(E, dtype=torch.int32, device="cuda")
    work = torch.zeros(A + E, 3, dtype=torch.int32, device="cuda")
    wc = torch.zeros(1, dtype=torch.int32, device="cuda")
    sa = L.alloc_act(max_rows, H, "cuda")
    h = L.alloc_act(max_rows, I, "cuda")
    y = torch.empty(max_rows, H, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    st = status.status()

    def f(i):
        ops.moe_route(logits, k, 0, None, 1, 1, 1.0, True, ids, wts)
        ops.moe_align(ids, 0, E, BN, perm, seg, work, wc)
        ops.moe_gather(x.q, x.sf, k, perm, sa.q, sa.sf)
        ops.gemm_mx_grouped(G.q, G.sf, U.q, U.sf, True, sa.q, sa.sf, work, wc, I, E, BN, h.q, h.sf, st)
        ops.gemm_mx_grouped(D.q, D.sf, None, None, True, h.q, h.sf, work, wc, H, E, BN, y, None, st)
        ops.moe_combine(y, perm, wts, k, None, None, out)

    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    active = int((torch.bincount(ids.flatten().long(), minlength=E) > 0).sum()) if a.reps else E
    wbytes = active * 3 * I * H * (0.5 + 1 / 32)
    return {"kernel": "moe_layer", "T": T, "E": E, "topk": k, "H": H, "I": I, "active_experts": active,
            "us": us, "weight_bytes": wbytes, "flops": 2.0 * A * 3 * I * H}


def bench_decode(a) -> dict:
    """Eager (graph-free) decode steps of a full model, each inside an NVTX range, so a launch list
    taken with ``ncu --nvtx --nvtx-include decode_step/`` covers exactly the decode kernels."""
    import numpy as np

    from ..engine.llm import LLM
    from ..engine.runner import pack_step
    from ..engine.scheduler import SamplingParams, ScheduledChunk, SchedulerOutput
    from ..models.config import EngineConfig, flashnext_moe, qwen27b_hybrid

    cfg = qwen27b_hybrid() if a.model == "dense27b" else flashnext_moe()
    if a.layers:
        cfg = cfg.scaled(layers=a.layers)
    ec = EngineConfig(max_batch=a.streams, max_model_len=a.prompt + 64, max_prefill_tokens=max(a.prompt, 256),
                      cuda_graphs=False)
    llm = LLM(cfg, ec, seed=0)
    rng = np.random.default_rng(0)
    seqs = [llm.add_request(rng.integers(0, cfg.vocab, a.prompt).tolist(), SamplingParams(max_tokens=32))
            for _ in range(a.streams)]
    while any(not s.prefill_done or not s.output for s in seqs):
        llm.step()
    for s in seqs:
        assert llm.scheduler.ensure(s, s.length + 1)
    out = SchedulerOutput("decode", [ScheduledChunk(s, s.length - 1, 1, True) for s in seqs])
    lay, arr = pack_step(out, ec.kv_block)
    llm.runner._upload(arr)
    meta = llm.runner.meta.views(lay)
    ws = llm.runner.ws

    def f(i):
        torch.cuda.nvtx.range_push("decode_step")
        llm.model.forward(meta, ws, lay.T, lay.R)
        torch.cuda.nvtx.range_pop()

    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    return {"kernel": "decode_step_eager", "model": cfg.name, "streams": a.streams, "layers": cfg.layers,
            "us": us, "weight_bytes": llm.model.weight_bytes(), "flops": 0.0}


def bench_prefill(a) -> dict:
    """One prompt of ``--prompt`` tokens prefilled through ``LLM.step()`` (all chunks of one step),
    device-timed with CUDA events after a warm-up prompt; ``--layers`` builds a shallower copy of the
    model (the per-layer time is reported so a full-depth figure can be scaled from it)."""
    import numpy as np

    from ..engine.llm import LLM
    from ..engine.scheduler import SamplingParams
    from ..models.config import EngineConfig, flashnext_moe, qwen27b_hybrid
    from ..models.mla_moe import glm53_flash

    full = {"dense27b": qwen27b_hybrid, "flashnext": flashnext_moe, "glm53": glm53_flash}[a.model]()
    cfg = full.scaled(layers=a.layers) if a.layers else full
    P = a.prompt
    ec = EngineConfig(max_batch=1, max_model_len=P + 64, max_prefill_tokens=P, cuda_graphs=False)
    llm = LLM(cfg, ec, seed=0)
    rng = np.random.default_rng(0)
    times = []
    for it in range(1 + a.reps):
        llm.add_request(rng.integers(0, cfg.vocab, P).tolist(), SamplingParams(max_tokens=1))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        while llm.has_unfinished():
            llm.step()
        e1.record()
        torch.cuda.synchronize()
        if it:
            times.append(e0.elapsed_time(e1))
    ms = min(times)
    return {"kernel": "prefill_step", "model": cfg.name, "prompt": P, "layers": cfg.layers, "full_layers": full.layers,
            "ms": ms, "tok_s": P / (ms / 1e3), "ms_per_layer": ms / cfg.layers,
            "full_depth_ms_est": ms / cfg.layers * full.layers, "us": ms * 1e3, "weight_bytes": 0.0, "flops": 0.0}


def bench_spec(a) -> dict:
    """Speculative verify steps (1 + k rows per sequence: forward, argmax, acceptance, GDN commit)
    through ``ModelRunner.execute_spec``, end to end on the host clock (metadata packing, upload,
    launch or graph replay, the token read-back), replayed from the verify CUDA graph and eagerly."""
    import time

    import numpy as np

    from ..engine.llm import LLM
    from ..engine.scheduler import SamplingParams, ScheduledChunk, SchedulerOutput
    from ..models.config import EngineConfig, flashnext_moe, qwen27b_hybrid

    full = qwen27b_hybrid() if a.model == "dense27b" else flashnext_moe()
    cfg = full.scaled(layers=a.layers) if a.layers else full
    ec = EngineConfig(max_batch=a.streams, max_model_len=a.prompt + 256, max_prefill_tokens=max(a.prompt, 256),
                      cuda_graphs=True, graph_batch_sizes=[1, 2, 4, 8, 16], spec_tokens=a.k, spec_method="ngram")
    llm = LLM(cfg, ec, seed=0)
    rng = np.random.default_rng(0)
    seqs = [llm.add_request(rng.integers(0, cfg.vocab, a.prompt).tolist(), SamplingParams(max_tokens=64))
            for _ in range(a.streams)]
    while any(not s.prefill_done or not s.output for s in seqs):
        out = llm.scheduler.schedule()
        llm.scheduler.finish_step(out, llm.runner.execute(out))
    for s in seqs:
        assert llm.scheduler.ensure(s, s.length + a.k + 1)
    out = SchedulerOutput("decode", [ScheduledChunk(s, s.length - 1, 1, True) for s in seqs])
    drafts = {s.seq_id: [1] * a.k for s in seqs}
    res = {}
    for mode in ("graph", "eager"):
        llm.runner.cfg.cuda_graphs = mode == "graph"
        for _ in range(a.warmup):
            llm.runner.execute_spec(out, drafts)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(a.reps):
            llm.runner.execute_spec(out, drafts)
        torch.cuda.synchronize()
        res[mode + "_us"] = (time.perf_counter() - t0) / a.reps * 1e6
    llm.runner.cfg.cuda_graphs = True
    return {"kernel": "spec_verify_step", "model": cfg.name, "layers": cfg.layers, "streams": a.streams, "k": a.k,
            **res, "graph_speedup": res["eager_us"] / res["graph_us"], "us": res["graph_us"],
            "weight_bytes": 0.0, "flops": 0.0}


def bench_gdn(a) -> dict:
    """The fused GDN decode kernel alone: S sequences, one token each; states rotate over enough
    layers' worth of buffers that every launch reads its state from HBM."""
    from .. import _native
    from ..utils import status

    torch.manual_seed(0)
    S, Hk, Hv, D = a.S, a.Hk, a.Hv, 128
    if a.prefill:
        return _bench_gdn_prefill(a)
    C = 2 * Hk * D + Hv * D
    rows = C + Hv * D + 2 * Hv
    sdt = torch.float32 if a.state == "fp32" else torch.bfloat16
    per = S * Hv * D * D * (4 if a.state == "fp32" else 2)
    nb = max(1, min(16, int(2 * L2_BYTES // per) + 1))
    states = [(torch.randn(S + 1, Hv, D, D, device="cuda") * 0.01).to(sdt) for _ in range(nb)]
    convs = [torch.randn(S + 1, C, 3, device="cuda").to(sdt) for _ in range(nb)]
    proj = torch.randn(S, rows, device="cuda").bfloat16()
    conv_w = (torch.randn(C, 4, device="cuda") * 0.3).bfloat16()
    A_log = torch.rand(Hv, device="cuda") * 2
    dt = torch.randn(Hv, device="cuda") * 0.5
    nw = torch.ones(D, device="cuda").bfloat16()
    slot = torch.arange(1, S + 1, dtype=torch.int32, device="cuda")
    hs = torch.ones(S, dtype=torch.int32, device="cuda")
    oq = torch.empty(S, Hv * D, dtype=torch.uint8, device="cuda")
    osf = torch.zeros(((S + 127) // 128 + 1) * 512 * (Hv * D // 128) + 4096, dtype=torch.uint8, device="cuda")
    ops = _native.ops()
    z_off = 2 * Hk * D + Hv * D
    f = lambda i: ops.gdn_decode_fused(proj, Hk, Hv, z_off, z_off + Hv * D, z_off + Hv * D + Hv, conv_w,
                                       convs[i % nb], states[i % nb], slot, hs, A_log, dt, nw, 1e-6, oq, osf, None)
    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    status.check()
    return {"kernel": "gdn_decode_fused", "S": S, "Hk": Hk, "Hv": Hv, "state": a.state, "us": us,
            "weight_bytes": 2.0 * per, "flops": 0.0}


def _bench_gdn_prefill(a) -> dict:
    """The token-serial delta-rule recurrence over a prefill: one sequence of ``--prefill`` tokens,
    Hv value heads (the conv / norm kernels around it are not included)."""
    from .. import _native

    T, Hk, Hv, D = a.prefill, a.Hk, a.Hv, 128
    nrm = lambda x: x / x.norm(dim=-1, keepdim=True)
    q = nrm(torch.randn(T, Hk, D, device="cuda")) * D ** -0.5
    k = nrm(torch.randn(T, Hk, D, device="cuda"))
    v = torch.randn(T, Hv, D, device="cuda")
    g = -torch.rand(T, Hv, device="cuda") * 0.5
    b = torch.rand(T, Hv, device="cuda")
    sdt = torch.float32 if a.state == "fp32" else torch.bfloat16
    st = torch.zeros(2, Hv, D, D, device="cuda", dtype=sdt)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")
    slot, s0, ln, hs = i32([1]), i32([0]), i32([T]), i32([0])
    o = torch.empty(T, Hv, D, device="cuda")
    ops = _native.ops()
    if a.chunked:
        from ..utils import status

        rows = [(j, min(128, T - j), 0) for j in range(0, T, 128)]
        ctab = torch.tensor(rows, dtype=torch.int32, device="cuda")
        c0 = i32([0, len(rows)])
        nr = len(rows) * Hv * 128
        buf = [torch.empty(nr, 128, dtype=torch.bfloat16, device="cuda") for _ in range(4)]
        buf += [torch.empty(nr, 128, device="cuda"), torch.empty(len(rows) * Hv, device="cuda")]
        stat = status.status(torch.device("cuda"))
        qkv = torch.cat([q, k, v], 1).bfloat16().contiguous()
        f = lambda i: ops.gdn_chunked(qkv, g, b, st, ctab, c0, slot, hs, True, Hk, Hv, *buf, o, stat)
        if a.trace:
            tr = torch.zeros(len(rows) * Hv * 8, dtype=torch.int64, device="cuda")
            ops.gdn_chunk_trace(tr)
            f(0)
            torch.cuda.synchronize()
            ops.gdn_chunk_trace(None)
            t = tr.view(-1, 8).cpu().double()
            t = t[t[:, 0] > 0]
            names = ("entry", "tiles", "mma1", "LP", "solve", "Ttiles", "mma2", "out")
            ph = {f"{names[i - 1]}->{names[i]}": round(float((t[:, i] - t[:, i - 1]).median()) / 1e3, 2)
                  for i in range(1, 8)}
            print(json.dumps({"gdn_phase1_median_us": ph, "ctas": int(t.shape[0]),
                              "span_us": round(float(t[:, 7].max() - t[:, 0].min()) / 1e3, 1)}))
    else:
        f = lambda i: ops.gdn_recurrent(q, k, v, g, b, st, slot, s0, ln, hs, True, o)
    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    return {"kernel": "gdn_chunked_prefill" if a.chunked else "gdn_recurrent_prefill", "T": T, "Hk": Hk, "Hv": Hv,
            "state": a.state, "us": us,
            "us_per_token": us / T, "weight_bytes": 0.0, "flops": 6.0 * T * Hv * D * D}


def bench_attn(a) -> dict:
    """tcgen05 split-KV decode attention over a paged fp8 KV cache: S sequences x ctx positions,
    hq / hkv heads of 256, one query token per sequence (the decode shape of the dense model)."""
    from .. import _native
    from ..utils import status

    torch.manual_seed(0)
    S, ctx, hq, hkv, D, BLK = a.S, a.ctx, a.hq, a.hkv, 256, 64
    nbps = (ctx + BLK - 1) // BLK
    nblk = S * nbps + 1
    kc = torch.randint(0, 255, (nblk, hkv, BLK, D), dtype=torch.uint8, device="cuda") & 0x7E
    vc = torch.randint(0, 255, (nblk, hkv, BLK, D), dtype=torch.uint8, device="cuda") & 0x7E
    bt = (torch.arange(S * nbps, dtype=torch.int32, device="cuda") + 1).view(S, nbps)
    q = torch.randn(S, hq, D, device="cuda").bfloat16()
    tok_ctx = torch.full((S,), ctx, dtype=torch.int32, device="cuda")
    st0 = torch.arange(S, dtype=torch.int32, device="cuda")
    ln = torch.ones(S, dtype=torch.int32, device="cuda")
    nsplit = a.nsplit or max(1, min(16, 148 // (S * hkv)))
    po = torch.empty(S * hq, nsplit, D, device="cuda")
    pml = torch.empty(S * hq, nsplit, 2, device="cuda")
    out = torch.empty(S, hq * D, dtype=torch.bfloat16, device="cuda")
    ops = _native.ops()
    stt = status.status()
    f = lambda i: ops.attn_tc_decode(q, kc, vc, bt, tok_ctx, st0, ln, D ** -0.5, 1.0, 1.0, po, pml, None, out, None,
                                     None, stt)
    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    kv_bytes = 2.0 * S * ctx * hkv * D
    return {"kernel": "attn_tc_decode", "S": S, "ctx": ctx, "hq": hq, "hkv": hkv, "nsplit": nsplit, "us": us,
            "weight_bytes": kv_bytes, "flops": 4.0 * S * hq * ctx * D}


def bench_qsa(a) -> dict:
    """QSA sparse decode attention (Flash-Next full-attention layers): S sequences at ctx positions,
    each attending to k selected 4-token groups + its open group's tail, hq / hkv heads of 256 over
    a paged fp8 KV cache. Bytes = the gathered K and V rows."""
    from .. import _native
    from ..utils import status

    torch.manual_seed(0)
    S, ctx, hq, hkv, D, BLK, K = a.S, a.ctx, a.hq, a.hkv, 256, 64, a.topk
    nbps = (ctx + BLK - 1) // BLK
    nblk = S * nbps + 1
    kc = torch.randint(0, 255, (nblk, hkv, BLK, D), dtype=torch.uint8, device="cuda") & 0x7E
    vc = torch.randint(0, 255, (nblk, hkv, BLK, D), dtype=torch.uint8, device="cuda") & 0x7E
    bt = (torch.arange(S * nbps, dtype=torch.int32, device="cuda") + 1).view(S, nbps)
    q = torch.randn(S, hq, D, device="cuda").bfloat16()
    tok_ctx = torch.full((S,), ctx, dtype=torch.int32, device="cuda")
    tok_seq = torch.arange(S, dtype=torch.int32, device="cuda")
    vis = ctx // 4
    sel = torch.stack([torch.randperm(vis, device="cuda")[:K].sort().values for _ in range(S)]).int()
    cnt = torch.full((S,), min(K, vis), dtype=torch.int32, device="cuda")
    nsplit = a.nsplit or max(1, min(16, -(-296 // (S * hkv))))
    po = torch.empty(S * hq, nsplit, D, device="cuda")
    pml = torch.empty(S * hq, nsplit, 2, device="cuda")
    gate = torch.randn(S, hq * D, device="cuda").bfloat16()
    out = torch.empty(S, hq * D, dtype=torch.bfloat16, device="cuda")
    ops = _native.ops()
    f = lambda i: ops.qsa_attention(q, kc, vc, bt, tok_seq, tok_ctx, sel, cnt, D ** -0.5, 1.0, 1.0, nsplit, po, pml,
                                    gate, out)
    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    status.check()
    keys = 4 * min(K, vis) + (ctx - 4 * vis)
    return {"kernel": "qsa_attention", "S": S, "ctx": ctx, "topk_groups": K, "hq": hq, "hkv": hkv, "nsplit": nsplit,
            "us": us, "weight_bytes": 2.0 * S * hkv * keys * D, "flops": 4.0 * S * hq * keys * D}


def bench_hc(a) -> dict:
    """Fused hyper-connection norm point: T rows, HC streams of H (bytes: residual read + write, the
    re-read of the second pass, block output, weights, gates and the mixed output)."""
    from ..models.weights import WeightFactory
    from ..ops import hc as HCo
    from ..utils import status

    T, HC, H = a.T, a.hc, a.H
    p = HCo.random_point(WeightFactory(torch.device("cuda"), seed=1, std=0.02), HC, H)
    res = torch.randn(T, HC * H, device="cuda").bfloat16()
    y = torch.randn(T, H, device="cuda").bfloat16()
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    f = lambda i: HCo.point(res, y, p, HC, 1e-6, out)
    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    status.check()
    nbytes = 2.0 * (3 * T * HC * H + 2 * T * H + 3 * HC * H)
    return {"kernel": "hc_point", "T": T, "HC": HC, "H": H, "us": us, "weight_bytes": nbytes, "flops": 0.0}


def bench_mla(a) -> dict:
    """Sparse MLA attention (GLM / DeepSeek-class): T query tokens of H heads, each attending to k
    selected latent rows (576 bf16 = 512 latent + 64 rope) of a paged cache at ctx positions, split
    over nsplit partials + the combine. ``--simple`` times the CUDA-core kernel instead of tcgen05.
    Bytes = the gathered rows; FLOPs = 2 T H k (576 + 512)."""
    from .. import _native
    from ..utils import status

    torch.manual_seed(0)
    T, H, ctx, K, BLK = a.T, a.H, a.ctx, a.topk, 64
    nbps = (ctx + BLK - 1) // BLK
    nblk = T * nbps + 1
    lat = (torch.randn(nblk, BLK, 576, device="cuda") * 0.5).bfloat16()
    bt = (torch.arange(T * nbps, dtype=torch.int32, device="cuda") + 1).view(T, nbps)
    tok_seq = torch.arange(T, dtype=torch.int32, device="cuda")
    n = min(K, ctx)
    sel = torch.stack([torch.randperm(ctx, device="cuda")[:n].sort().values for _ in range(T)]).int()
    cnt = torch.full((T,), n, dtype=torch.int32, device="cuda")
    q = torch.randn(T, H, 576, device="cuda").bfloat16()
    nsplit = a.nsplit or 4
    po = torch.empty(T * H, nsplit, 512, device="cuda")
    pml = torch.empty(T * H, nsplit, 2, device="cuda")
    out = torch.empty(T, H, 512, dtype=torch.bfloat16, device="cuda")
    ops, st = _native.ops(), status.status(torch.device("cuda"))
    if a.indexer:
        # lightning-indexer scores over the whole context (R9K_INDEXER=simple: the CUDA-core kernel)
        Hi = 32
        ic = torch.randint(0, 255, (nblk, BLK, 128), dtype=torch.uint8, device="cuda") & 0x7E
        qi = torch.randn(T, Hi, 128, device="cuda").bfloat16()
        wi = torch.rand(T, Hi, device="cuda")
        ctxs = torch.full((T,), ctx, dtype=torch.int32, device="cuda")
        sc = torch.empty(T, ctx, device="cuda")
        f = lambda i: ops.indexer_score(qi, wi, ic, bt, tok_seq, ctxs, ctx, sc, st)
        us = _time(f, a.reps, a.warmup, graph=not a.eager)
        status.check()
        import os

        return {"kernel": "indexer_score_" + os.environ.get("R9K_INDEXER", "tc"), "T": T, "Hi": Hi, "ctx": ctx,
                "us": us, "weight_bytes": 128.0 * T * ctx, "flops": 2.0 * T * Hi * ctx * 128}
    if a.simple:
        f = lambda i: ops.sparse_mla_decode(q, lat, bt, tok_seq, sel, cnt, 192 ** -0.5, po, pml, out)
    else:
        f = lambda i: ops.sparse_mla_decode_tc(q, lat, bt, tok_seq, sel, cnt, 192 ** -0.5, po, pml, out, st)
    us = _time(f, a.reps, a.warmup, graph=not a.eager)
    status.check()
    return {"kernel": "sparse_mla_decode" + ("" if a.simple else "_tc"), "T": T, "H": H, "ctx": ctx, "topk": n,
            "nsplit": nsplit, "us": us, "weight_bytes": 1152.0 * T * n, "flops": 2.0 * T * H * n * (576 + 512)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--N", type=int, default=5120)
    g.add_argument("--K", type=int, default=17408)
    g.add_argument("--M", type=int, default=16)
    g.add_argument("--fmt", choices=["fp4", "fp8", "bf16"], default="fp4")
    g.add_argument("--swiglu", action="store_true")
    g.add_argument("--tiled", type=int, default=1)
    g.add_argument("--max-copies", type=int, default=16)
    g.add_argument("--vs-torch", action="store_true", help="bf16: also time torch.matmul (cuBLAS) on the same weights")
    g.add_argument("--trace", action="store_true", help="per-CTA phase timestamps of the last launch (gemm_trace)")
    m = sub.add_parser("moe")
    m.add_argument("--T", type=int, default=16)
    m.add_argument("--E", type=int, default=288)
    m.add_argument("--topk", type=int, default=10)
    m.add_argument("--H", type=int, default=2048)
    m.add_argument("--I", type=int, default=512)
    d = sub.add_parser("decode")
    d.add_argument("--model", choices=["dense27b", "flashnext"], default="dense27b")
    d.add_argument("--streams", type=int, default=16)
    d.add_argument("--prompt", type=int, default=256)
    d.add_argument("--layers", type=int, default=0)
    pf = sub.add_parser("prefill")
    pf.add_argument("--model", choices=["dense27b", "flashnext", "glm53"], default="glm53")
    pf.add_argument("--prompt", type=int, default=8192)
    pf.add_argument("--layers", type=int, default=0)
    sp = sub.add_parser("spec")
    sp.add_argument("--model", choices=["dense27b", "flashnext"], default="dense27b")
    sp.add_argument("--layers", type=int, default=0)
    sp.add_argument("--streams", type=int, default=16)
    sp.add_argument("--prompt", type=int, default=256)
    sp.add_argument("--k", type=int, default=3)
    gd = sub.add_parser("gdn")
    gd.add_argument("--S", type=int, default=16)
    gd.add_argument("--Hk", type=int, default=16)
    gd.add_argument("--Hv", type=int, default=48)
    gd.add_argument("--state", choices=["bf16", "fp32"], default="bf16")
    gd.add_argument("--prefill", type=int, default=0, help="time the prefill recurrence over this many tokens")
    gd.add_argument("--chunked", action="store_true", help="with --prefill: the tcgen05 chunked kernels")
    gd.add_argument("--trace", action="store_true", help="with --chunked: phase-1 timestamps")
    at = sub.add_parser("attn")
    at.add_argument("--S", type=int, default=16)
    at.add_argument("--ctx", type=int, default=8192)
    at.add_argument("--hq", type=int, default=24)
    at.add_argument("--hkv", type=int, default=4)
    at.add_argument("--nsplit", type=int, default=0)
    qs = sub.add_parser("qsa")
    qs.add_argument("--S", type=int, default=16)
    qs.add_argument("--ctx", type=int, default=8192)
    qs.add_argument("--hq", type=int, default=16)
    qs.add_argument("--hkv", type=int, default=2)
    qs.add_argument("--topk", type=int, default=512)
    qs.add_argument("--nsplit", type=int, default=0)
    ml = sub.add_parser("mla")
    ml.add_argument("--T", type=int, default=16)
    ml.add_argument("--H", type=int, default=64)
    ml.add_argument("--ctx", type=int, default=8192)
    ml.add_argument("--topk", type=int, default=2048)
    ml.add_argument("--nsplit", type=int, default=0)
    ml.add_argument("--simple", action="store_true", help="the CUDA-core kernel")
    ml.add_argument("--indexer", action="store_true", help="time the indexer scores instead (32 heads, whole context)")
    hcp = sub.add_parser("hc")
    hcp.add_argument("--T", type=int, default=16)
    hcp.add_argument("--hc", type=int, default=4)
    hcp.add_argument("--H", type=int, default=2048)
    for p in (g, m, d, pf, sp, gd, at, qs, ml, hcp):
        p.add_argument("--eager", action="store_true", help="time eager launches (host overhead included)")
        p.add_argument("--reps", type=int, default=50)
        p.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args(argv)
    r = {"gemm": bench_gemm, "moe": bench_moe, "decode": bench_decode, "prefill": bench_prefill, "spec": bench_spec,
         "gdn": bench_gdn,
         "attn": bench_attn,
         "qsa": bench_qsa, "mla": bench_mla, "hc": bench_hc}[a.cmd](a)
    pk = peaks()
    if r["us"] > 0:
        r["gbs"] = r["weight_bytes"] / r["us"] / 1e3
        r["tflops"] = r["flops"] / r["us"] / 1e6
        r["frac_hbm"] = round(r["gbs"] / pk["hbm_gbs"], 3)
        r["frac_bf16"] = round(r["tflops"] / pk["bf16_tflops"], 4)
        r["peaks"] = pk["src"]
    print(json.dumps(r))
    return r


if __name__ == "__main__":
    main()
