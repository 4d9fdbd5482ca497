"""MoE kernels (routing, alignment, grouped GEMMs, combine) and the MoE model vs plain PyTorch."""
import pytest
import torch
import torch.nn.functional as Fn

pytestmark = pytest.mark.gpu


def _ops():
    from r9700_stack_b200 import _native

    return _native.ops()


def _check():
    from r9700_stack_b200.utils import status

    torch.cuda.synchronize()
    status.check()


def test_route_softmax_topk():
    torch.manual_seed(0)
    T, E, k = 37, 288, 10
    logits = torch.randn(T, E).cuda()
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    w = torch.empty(T, k, device="cuda")
    _ops().moe_route(logits, k, 0, None, 1, 1, 1.0, True, ids, w)
    _check()
    p = torch.softmax(logits, -1)
    rw, rid = torch.topk(p, k, -1)
    assert torch.equal(ids.long().sort(-1).values, rid.sort(-1).values)
    torch.testing.assert_close(w.sort(-1).values, (rw / rw.sum(-1, keepdim=True)).sort(-1).values)


def test_route_sigmoid_grouped():
    torch.manual_seed(1)
    T, E, k, G, TG = 20, 256, 8, 8, 4
    logits = torch.randn(T, E).cuda()
    bias = (torch.randn(E) * 0.1).cuda()
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    w = torch.empty(T, k, device="cuda")
    _ops().moe_route(logits, k, 1, bias, G, TG, 2.5, True, ids, w)
    _check()
    s = torch.sigmoid(logits)
    b = s + bias
    gs = b.view(T, G, -1).topk(2, -1).values.sum(-1)
    keep = torch.zeros(T, G, dtype=torch.bool, device="cuda").scatter_(1, gs.topk(TG, -1).indices, True)
    b = b.masked_fill(~keep.repeat_interleave(E // G, 1), float("-inf"))
    rid = b.topk(k, -1).indices
    rw = s.gather(1, rid)
    rw = rw / rw.sum(-1, keepdim=True) * 2.5
    assert torch.equal(ids.long().sort(-1).values, rid.sort(-1).values)
    torch.testing.assert_close(w.sort(-1).values, rw.sort(-1).values)


@pytest.mark.parametrize("T,BN", [(5, 16), (40, 128), (40, 16), (60, 32), (90, 64)])
def test_grouped_experts_match_torch(T, BN):
    from r9700_stack_b200.ops import linear as L
    from r9700_stack_b200.quant import formats as F

    torch.manual_seed(2)
    E, k, H, I = 6, 2, 256, 256
    ws_g = [L.mx_from_float((torch.randn(I, H) * 0.05).cuda()) for _ in range(E)]
    ws_u = [L.mx_from_float((torch.randn(I, H) * 0.05).cuda()) for _ in range(E)]
    ws_d = [L.mx_from_float((torch.randn(H, I) * 0.05).cuda()) for _ in range(E)]
    G, U, D = L.stack_experts(ws_g), L.stack_experts(ws_u), L.stack_experts(ws_d)
    x = torch.randn(T, H).bfloat16().cuda()
    ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).int().cuda()
    w = torch.rand(T, k).cuda()
    A = T * k
    max_rows = A + 256 * min(E, A)
    perm = torch.empty(A, dtype=torch.int32, device="cuda")
    seg = torch.empty(E, dtype=torch.int32, device="cuda")
    work = torch.zeros(A + E, 3, dtype=torch.int32, device="cuda")
    wc = torch.zeros(1, dtype=torch.int32, device="cuda")
    o = _ops()
    o.moe_align(ids, 0, E, BN, perm, seg, work, wc)
    xa = L.quant_act(x)
    sa = L.alloc_act(max_rows, H, "cuda")
    o.moe_gather(xa.q, xa.sf, k, perm, sa.q, sa.sf)
    h = L.alloc_act(max_rows, I, "cuda")
    from r9700_stack_b200.utils import status
    st = status.status()
    o.gemm_mx_grouped(G.q, G.sf, U.q, U.sf, True, sa.q, sa.sf, work, wc, I, E, BN, h.q, h.sf, st)
    y = torch.zeros(max_rows, H, dtype=torch.bfloat16, device="cuda")
    o.gemm_mx_grouped(D.q, D.sf, None, None, True, h.q, h.sf, work, wc, H, E, BN, y, None, st)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    o.moe_combine(y, perm, w, k, None, None, out)
    _check()
    xq = F.dequant_mx(xa.q.cpu(), xa.sf.cpu(), T, H, False).cuda()
    ref = torch.zeros(T, H, device="cuda")
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            hh = Fn.silu(xq[t] @ ws_g[e].dequant().T) * (xq[t] @ ws_u[e].dequant().T)
            from r9700_stack_b200.models.reference import fake_mxfp8
            ref[t] += w[t, j] * (fake_mxfp8(hh[None])[0] @ ws_d[e].dequant().T).bfloat16().float()
    torch.testing.assert_close(out.float(), ref, rtol=3e-2, atol=3e-2 * float(ref.abs().max()))


def test_tiny_moe_model_matches_reference():
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_moe
    from r9700_stack_b200.models.reference import ReferenceState, reference_forward

    cfg = tiny_moe(gdn_state_dtype="fp32")
    ec = EngineConfig(max_batch=2, max_model_len=256, max_prefill_tokens=128, cuda_graphs=True,
                      graph_batch_sizes=[1, 2])
    llm = LLM(cfg, ec, seed=4)
    prompt = list(range(5, 45))
    seq = llm.add_request(prompt, SamplingParams(max_tokens=3))
    st = ReferenceState(llm.model)
    llm.step()
    _check()
    got = llm.runner.ws.logits[0].clone()
    ref = reference_forward(llm.model, prompt, st)[-1]
    cos = torch.nn.functional.cosine_similarity(got.double(), ref.double(), dim=0)
    assert float(cos) > 0.99, float(cos)
    llm.step()
    _check()
    got = llm.runner.ws.logits[0].clone()
    ref = reference_forward(llm.model, [seq.output[-2]], st)[-1]
    cos = torch.nn.functional.cosine_similarity(got.double(), ref.double(), dim=0)
    assert float(cos) > 0.99, float(cos)


@pytest.mark.parametrize("T,k,E,e0,El,BN", [(16, 10, 288, 0, 288, 16), (3000, 8, 256, 64, 128, 128), (7, 2, 8, 0, 8, 16),
                                            (64, 10, 8, 0, 8, 16), (200, 4, 16, 0, 16, 32)])
def test_align_matches_python(T, k, E, e0, El, BN):
    torch.manual_seed(T)
    ids = torch.randint(0, E, (T, k), dtype=torch.int32)
    A = T * k
    perm = torch.empty(A, dtype=torch.int32, device="cuda")
    seg = torch.empty(El, dtype=torch.int32, device="cuda")
    max_work = A + El
    work = torch.zeros(max_work, 3, dtype=torch.int32, device="cuda")
    wc = torch.zeros(1, dtype=torch.int32, device="cuda")
    _ops().moe_align(ids.cuda(), e0, El, BN, perm, seg, work, wc)
    _check()
    flat = ids.flatten().tolist()
    cnt = [0] * El
    for e in flat:
        if e0 <= e < e0 + El:
            cnt[e - e0] += 1
    # every work item starts on a 128-row boundary: with BN < 128 one 128-row slot per BN rows
    stride = BN if BN >= 128 else 128
    start, s = [], 0
    for c in cnt:
        start.append(s)
        s += (c + 127) // 128 * 128 if BN >= 128 else (c + BN - 1) // BN * 128
    ref_perm, cur = [], [0] * El
    for e in flat:
        if e0 <= e < e0 + El:
            r = cur[e - e0]
            ref_perm.append(start[e - e0] + (r if BN >= 128 else (r // BN) * 128 + r % BN))
            cur[e - e0] += 1
        else:
            ref_perm.append(-1)
    assert perm.cpu().tolist() == ref_perm
    assert seg.cpu().tolist() == start
    ref_work = [[e, start[e] + i * stride, min(BN, cnt[e] - i * BN)] for e in range(El)
                for i in range((cnt[e] + BN - 1) // BN)]
    assert int(wc) == len(ref_work)
    assert work[: len(ref_work)].cpu().tolist() == ref_work


def test_tiny_moe_with_ple_matches_reference():
    """Per-layer embeddings from the pinned-host int6 table (Flash-Next class) vs the oracle."""
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_moe
    from r9700_stack_b200.models.reference import ReferenceState, reference_forward

    cfg = tiny_moe(gdn_state_dtype="fp32", ple_dim=64)
    ec = EngineConfig(max_batch=2, max_model_len=256, max_prefill_tokens=128, graph_batch_sizes=[1, 2])
    llm = LLM(cfg, ec, seed=4)
    assert llm.model.ple is not None
    prompt = list(range(5, 30))
    seq = llm.add_request(prompt, SamplingParams(max_tokens=3))
    st = ReferenceState(llm.model)
    llm.step()
    _check()
    got = llm.runner.ws.logits[0].clone()
    ref = reference_forward(llm.model, prompt, st)[-1]
    cos = torch.nn.functional.cosine_similarity(got.double(), ref.double(), dim=0)
    assert float(cos) > 0.99, float(cos)
    llm.step()
    _check()
    got = llm.runner.ws.logits[0].clone()
    ref = reference_forward(llm.model, [seq.output[-2]], st)[-1]
    cos = torch.nn.functional.cosine_similarity(got.double(), ref.double(), dim=0)
    assert float(cos) > 0.99, float(cos)


def test_expert_placement_is_the_same_function(tmp_path):
    """A tiny MoE model under two expert placements (different local orders) gives identical logits,
    and matches the fp32 oracle."""
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_moe
    from r9700_stack_b200.models.reference import ReferenceState, reference_forward
    from r9700_stack_b200.parallel import ep_placement as P

    cfg = tiny_moe(gdn_state_dtype="fp32")
    outs = []
    for perm in ([0, 1, 2, 3, 4, 5, 6, 7], [5, 2, 7, 0, 3, 6, 1, 4]):
        f = tmp_path / f"p{perm[0]}.json"
        P.save(str(f), [perm])
        ec = EngineConfig(max_batch=2, max_model_len=256, max_prefill_tokens=128, cuda_graphs=False,
                          ep_placement=str(f))
        llm = LLM(cfg, ec, seed=4)
        prompt = torch.randint(0, cfg.vocab, (24,), generator=torch.Generator().manual_seed(2)).tolist()
        llm.add_request(prompt, SamplingParams(max_tokens=2))
        llm.step()
        torch.cuda.synchronize()
        got = llm.runner.ws.logits[0].clone()
        outs.append(got)
        ref = reference_forward(llm.model, prompt, ReferenceState(llm.model))[-1]
        cos = float(torch.nn.functional.cosine_similarity(got.double(), ref.double(), dim=0))
        assert cos > 0.995, cos
    assert torch.equal(outs[0], outs[1])
