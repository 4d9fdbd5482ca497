"""Speculative decoding: the GDN commit and accept kernels vs PyTorch / the plain kernels, and
lossless greedy decoding through every drafter (outputs equal to non-speculative decoding)."""
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


@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
def test_gdn_spec_commit_matches_recurrent(state_dtype):
    torch.manual_seed(0)
    Hk, Hv, d, W = 2, 4, 128, 4
    C = 2 * Hk * d + Hv * d
    proj_rows = C + Hv * d + 2 * Hv
    n_per = [5, 3, 9]
    acc = [2, 3, 1]
    S, T = len(n_per), sum(n_per)
    starts = [0, 5, 8]
    slots = [3, 1, 2]
    layers = []
    for _ in range(2):
        lay = dict(
            k=torch.nn.functional.normalize(torch.randn(T, Hk, d), dim=-1).cuda(),
            v=torch.randn(T, Hv, d).cuda(),
            g=(-torch.rand(T, Hv)).cuda(),
            b=torch.rand(T, Hv).cuda(),
            proj=torch.randn(T, proj_rows).bfloat16().cuda(),
            ssm=(torch.randn(4, Hv, d, d) * 0.1).to(state_dtype).cuda(),
            conv=torch.randn(4, C, W - 1).to(state_dtype).cuda(),
        )
        layers.append(lay)
    ref = [(l["ssm"].clone(), l["conv"].clone()) for l in layers]
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")
    seq_slot, seq_start, acc_len, hs = i32(slots), i32(starts), i32(acc), i32([1, 1, 0])
    o = _ops()
    for l, (ssm, conv) in zip(layers, ref):
        q = torch.zeros(T, Hk, d, device="cuda")
        o.gdn_recurrent(q, l["k"], l["v"], l["g"], l["b"], ssm, seq_slot, seq_start, acc_len, hs, True, None)
        o.gdn_conv_state_update(l["proj"], conv, seq_slot, seq_start, acc_len, hs)
    table = torch.tensor([[l["k"].data_ptr(), l["v"].data_ptr(), l["g"].data_ptr(), l["b"].data_ptr(),
                           l["proj"].data_ptr(), l["ssm"].data_ptr(), l["conv"].data_ptr(), 0] for l in layers],
                         dtype=torch.int64).cuda()
    o.gdn_spec_commit(table, Hk, Hv, d, C, W, proj_rows, state_dtype == torch.float32, seq_slot, seq_start, acc_len, hs)
    _check()
    for l, (ssm, conv) in zip(layers, ref):
        torch.testing.assert_close(l["ssm"].float(), ssm.float(), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(l["conv"].float(), conv.float(), rtol=0, atol=0)


def test_spec_accept():
    ids = torch.tensor([5, 1, 2, 3, 7, 9, 4, 8, 8], dtype=torch.int32, device="cuda")
    tgt = torch.tensor([1, 2, 6, 0, 9, 1, 8, 8, 2], dtype=torch.int64, device="cuda")
    start = torch.tensor([0, 4, 6], dtype=torch.int32, device="cuda")
    ln = torch.tensor([4, 2, 3], dtype=torch.int32, device="cuda")
    acc = torch.zeros(3, dtype=torch.int32, device="cuda")
    _ops().spec_accept(ids, tgt, start, ln, acc)
    _check()
    # seq0: drafts 1,2,3 vs targets 1,2,6 -> 2 accepted; seq1: draft 9 vs 9 -> 1; seq2: 8,8 vs 8,8 -> 2
    assert acc.tolist() == [3, 2, 3]


def _engine(cfg, k=0, method="ngram", drafter=None, graphs=True):
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.models.config import EngineConfig

    ec = EngineConfig(max_batch=3, max_model_len=256, max_prefill_tokens=64, cuda_graphs=graphs,
                      graph_batch_sizes=[1, 2, 4], spec_tokens=k, spec_method=method)
    return LLM(cfg, ec, seed=7, drafter=drafter)


def _prompts():
    g = torch.Generator().manual_seed(3)
    return [torch.randint(1, 500, (n,), generator=g).tolist() for n in (37, 80, 12)]


@pytest.fixture(scope="module")
def greedy_ref():
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import tiny_hybrid

    llm = _engine(tiny_hybrid(gdn_state_dtype="fp32"))
    outs = llm.generate(_prompts(), SamplingParams(max_tokens=20))
    _check()
    return outs


def _agree(a, b):
    """Length of the common prefix (fp reduction order differs between the verify and decode
    shapes, so a rare near-tie may flip; the prefix must still be long)."""
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


@pytest.mark.parametrize("corrupt", [0, 3])
def test_spec_scripted_is_lossless(greedy_ref, corrupt):
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import tiny_hybrid
    from r9700_stack_b200.spec.drafters import ScriptedDrafter

    cfg = tiny_hybrid(gdn_state_dtype="fp32")
    dr = ScriptedDrafter(4, {}, pad=0, corrupt_every=corrupt)
    llm = _engine(cfg, k=4, drafter=dr)
    seqs = [llm.add_request(p, SamplingParams(max_tokens=20)) for p in _prompts()]
    for s, ref in zip(seqs, greedy_ref):
        dr.script[s.seq_id] = ref
    while llm.has_unfinished():
        llm.step()
    _check()
    for s, ref in zip(seqs, greedy_ref):
        assert _agree(s.output, ref) >= 16, (s.output, ref)
    st = llm.spec_stats
    if corrupt == 0:
        assert st["accepted"] >= 0.8 * st["drafted"], st
    else:
        assert 0 < st["accepted"] < st["drafted"], st


@pytest.mark.parametrize("method", ["ngram", "mtp", "block", "dspark"])
def test_spec_drafters_lossless(greedy_ref, method):
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import tiny_hybrid

    llm = _engine(tiny_hybrid(gdn_state_dtype="fp32"), k=3, method=method)
    outs = llm.generate(_prompts(), SamplingParams(max_tokens=20))
    _check()
    for o, ref in zip(outs, greedy_ref):
        assert len(o) == 20
        assert _agree(o, ref) >= 16, (o, ref)
    assert llm.spec_stats["steps"] > 0


def test_spec_moe_mtp_runs():
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import tiny_moe

    cfg = tiny_moe(gdn_state_dtype="fp32")
    ref = _engine(cfg).generate(_prompts(), SamplingParams(max_tokens=12))
    llm = _engine(cfg, k=3, method="mtp")
    outs = llm.generate(_prompts(), SamplingParams(max_tokens=12))
    _check()
    for o, r in zip(outs, ref):
        assert _agree(o, r) >= 9, (o, r)


def test_dspark_adaptive_lengths():
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import tiny_hybrid

    llm = _engine(tiny_hybrid(gdn_state_dtype="fp32"), k=4, method="dspark")
    llm.drafter.min_conf = 0.5  # random heads: confidence ~ sigmoid(small) -> some drafts are cut
    llm.generate(_prompts(), SamplingParams(max_tokens=10))
    _check()
    st = llm.spec_stats
    assert st["steps"] > 0 and 0 < st["drafted"] < st["steps"] * 3 * 4 + 1
    assert all(1 <= n <= 4 for n in llm.drafter.last_lengths)


def test_dspark_markov_kernel_matches_torch():
    """The one-launch-per-position Markov refinement (argmax over the vocabulary, confidence head,
    kept lengths) against the same refinement in torch ops with fp32 logits, two rounds in a row
    (the launch re-arms its own arrival counter)."""
    from r9700_stack_b200.models.config import tiny_hybrid

    llm = _engine(tiny_hybrid(gdn_state_dtype="fp32"), k=4, method="dspark")
    dr = llm.drafter
    dr.min_conf = 0.5
    g = torch.Generator(device="cuda").manual_seed(9)
    S, km, V = 3, 4, dr.vocab
    H = dr.conf_w.w.shape[1] - dr.markov_embed.shape[1]
    for _ in range(2):
        base = torch.randn(S, km, V, device="cuda", generator=g)
        hrows = torch.randn(S, km, H, device="cuda", generator=g).bfloat16()
        prev = torch.randint(0, V, (S,), device="cuda", generator=g)
        got = dr.refine(base, hrows, prev)
        want = dr.refine_reference(base, hrows, prev)
        _check()
        assert got == want, (got, want)
