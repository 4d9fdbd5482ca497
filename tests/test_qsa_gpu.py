"""QSA sparse attention: the gather-attention kernel against a masked fp32 softmax, the group key
compression against torch, and a tiny QSA model against the fp32 oracle (sparse regime: the
selection is smaller than the context)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from r9700_stack_b200 import _native

    return _native.ops()


def _check():
    from r9700_stack_b200.utils import status

    torch.cuda.synchronize()
    status.check()


def _f8(x):
    return x.view(torch.float8_e4m3fn).float()


@pytest.mark.parametrize("heads", [(16, 2), (4, 1), (12, 1)])
@pytest.mark.parametrize("nsplit", [1, 3])
def test_qsa_attention_matches_masked_softmax(heads, nsplit):
    torch.manual_seed(0)
    hq, hkv = heads
    D, BLK, K = 256, 64, 6
    ctxs = [7, 70, 200, 131]
    S = len(ctxs)
    nblocks = 24
    kc = (torch.randn(nblocks, hkv, BLK, D) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8).cuda()
    vc = torch.randn(nblocks, hkv, BLK, D).to(torch.float8_e4m3fn).view(torch.uint8).cuda()
    perm = torch.randperm(nblocks)
    bt = torch.zeros(S, 4, dtype=torch.int32)
    for s in range(S):
        bt[s] = perm[4 * s: 4 * s + 4]
    # one query row per sequence at its last position, plus a second row earlier in seq 2
    rows = [(s, c) for s, c in enumerate(ctxs)] + [(2, 150)]
    T = len(rows)
    tok_seq = torch.tensor([r[0] for r in rows], dtype=torch.int32)
    tok_ctx = torch.tensor([r[1] for r in rows], dtype=torch.int32)
    sel = torch.full((T, K), -1, dtype=torch.int32)
    cnt = torch.zeros(T, dtype=torch.int32)
    for t, (s, c) in enumerate(rows):
        vis = c // 4
        g = torch.randperm(vis)[: min(K, vis)].sort().values if vis > K else torch.arange(vis)
        sel[t, : len(g)] = g.int()
        cnt[t] = len(g)
    q = torch.randn(T, hq, D).bfloat16()
    gate = torch.randn(T, hq * D).bfloat16()
    out = torch.zeros(T, hq * D, dtype=torch.bfloat16).cuda()
    po = torch.zeros(T * hq, nsplit, D).cuda()
    pml = torch.zeros(T * hq, nsplit, 2).cuda()
    scale, ks, vs = D ** -0.5, 0.7, 1.3
    _ops().qsa_attention(q.cuda(), kc, vc, bt.cuda(), tok_seq.cuda(), tok_ctx.cuda(), sel.cuda(), cnt.cuda(),
                         scale, ks, vs, nsplit, po, pml, gate.cuda(), out)
    _check()
    G = hq // hkv
    for t, (s, c) in enumerate(rows):
        vis = c // 4
        keys = [4 * int(g) + j for g in sel[t, : cnt[t]] for j in range(4)] + list(range(4 * vis, c))
        tok = torch.tensor(keys)
        blk = bt[s][tok // 64].long()
        off = tok % 64
        for h in range(hq):
            kv = h // G
            Kf = _f8(kc.cpu()[blk, kv, off]) * ks
            Vf = _f8(vc.cpu()[blk, kv, off]) * vs
            p = torch.softmax((q[t, h].float() @ Kf.T) * scale, -1)
            ref = (p @ Vf) * torch.sigmoid(gate[t, h * D:(h + 1) * D].float())
            got = out[t, h * D:(h + 1) * D].float().cpu()
            assert torch.allclose(got, ref, atol=2e-2, rtol=2e-2), (t, h, (got - ref).abs().max())


def test_qsa_compress_means_token_keys():
    torch.manual_seed(1)
    nblocks, S = 8, 2
    ktok = (torch.randn(nblocks, 64, 128) * 0.5).bfloat16().cuda()
    ckey = torch.zeros(nblocks, 64, 128, dtype=torch.uint8).cuda()
    bt = torch.tensor([[3, 5, 1, 0], [2, 7, 4, 6]], dtype=torch.int32).cuda()
    tok_ctx = torch.tensor([4, 8, 130, 7, 256], dtype=torch.int32).cuda()
    tok_seq = torch.tensor([0, 0, 1, 1, 0], dtype=torch.int32).cuda()
    _ops().qsa_compress(ktok, bt, tok_seq, tok_ctx, ckey)
    _check()
    for c, s in zip(tok_ctx.tolist(), tok_seq.tolist()):
        if c % 4:
            continue
        g = c // 4 - 1
        toks = torch.arange(4 * g, 4 * g + 4)
        rows = ktok[bt[s][toks // 64].long(), toks % 64].float()
        ref = (rows.sum(0) * 0.25).to(torch.float8_e4m3fn).float()
        got = _f8(ckey[bt[s][g // 64], g % 64])
        assert torch.equal(got.cpu(), ref.cpu()), (c, s)


@pytest.mark.parametrize("graphs", [False, True])
def test_tiny_qsa_model_matches_reference(graphs):
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_hybrid
    from r9700_stack_b200.models.reference import ReferenceState, reference_forward

    cfg = tiny_hybrid(gdn_state_dtype="fp32", qsa_topk=4)
    ec = EngineConfig(max_batch=2, max_model_len=512, max_prefill_tokens=256, cuda_graphs=graphs,
                      graph_batch_sizes=[1, 2])
    llm = LLM(cfg, ec, seed=3)
    prompt = torch.randint(0, cfg.vocab, (70,), generator=torch.Generator().manual_seed(5)).tolist()
    seq = llm.add_request(prompt, SamplingParams(max_tokens=6))
    st = ReferenceState(llm.model)
    llm.step()  # prefill: 70 tokens, top-4 groups of up to 17 -> sparse
    _check()
    cos = lambda a, b: float(torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))
    got = llm.runner.ws.logits[0].clone()
    ref = reference_forward(llm.model, prompt, st)[-1]
    assert cos(got, ref) > 0.995, cos(got, ref)
    for _ in range(5):
        llm.step()
        _check()
        got = llm.runner.ws.logits[0].clone()
        ref = reference_forward(llm.model, [seq.output[-2]], st)[-1]
        assert cos(got, ref) > 0.99, cos(got, ref)
