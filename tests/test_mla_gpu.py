"""MLA + lightning indexer + top-k kernels vs plain PyTorch (GLM / DeepSeek sparse attention)."""
import math

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


def _rope_ref(x, pos, cs):
    c, s = cs[pos, :32], cs[pos, 32:]
    a, b = x[..., :32], x[..., 32:64]
    return torch.cat([a * c - b * s, b * c + a * s, x[..., 64:]], -1)


def _setup(ctxs, seed=0):
    torch.manual_seed(seed)
    BLK = 64
    nblk = sum((c + BLK - 1) // BLK for c in ctxs) + 1
    mb = max((c + BLK - 1) // BLK for c in ctxs)
    perm = (torch.randperm(nblk - 1) + 1).tolist()
    bt = torch.zeros(len(ctxs), mb, dtype=torch.int32)
    for s, c in enumerate(ctxs):
        for b in range((c + BLK - 1) // BLK):
            bt[s, b] = perm.pop()
    inv = 1.0 / (10000 ** (torch.arange(0, 64, 2, dtype=torch.float64) / 64))
    f = torch.outer(torch.arange(max(ctxs) + 8, dtype=torch.float64), inv)
    cs = torch.cat([f.cos(), f.sin()], -1).float().cuda()
    return nblk, bt.cuda(), cs


def test_cache_write_indexer_topk_and_sparse_attention():
    ctxs = [70, 300, 5]
    nblk, bt, cs = _setup(ctxs)
    o = _ops()
    # write every position of every sequence
    seqs, poss = [], []
    for s, c in enumerate(ctxs):
        seqs += [s] * c
        poss += list(range(c))
    T = len(seqs)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")
    slots = i32([int(bt[s, p // 64]) * 64 + p % 64 for s, p in zip(seqs, poss)])
    kv = torch.randn(T, 576).bfloat16().cuda()
    kvw = (1 + 0.1 * torch.randn(512)).bfloat16().cuda()
    ik = torch.randn(T, 128).bfloat16().cuda()
    ikw = (1 + 0.1 * torch.randn(128)).bfloat16().cuda()
    lat = torch.zeros(nblk, 64, 576, dtype=torch.bfloat16, device="cuda")
    icache = torch.zeros(nblk, 64, 128, dtype=torch.uint8, device="cuda")
    o.mla_cache_write(kv, kvw, ik, ikw, 1e-6, i32(poss), cs, slots, lat, icache)
    _check()
    posT = torch.tensor(poss, device="cuda")
    c = kv[:, :512].float()
    c = c * torch.rsqrt(c.square().mean(-1, keepdim=True) + 1e-6) * kvw.float()
    kpe = _rope_ref(kv[:, 512:].float(), posT, cs)
    got = lat.view(-1, 576)[slots.long()].float()
    torch.testing.assert_close(got[:, :512], c, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(got[:, 512:], kpe, rtol=1e-2, atol=1e-2)
    kk = ik.float() * torch.rsqrt(ik.float().square().mean(-1, keepdim=True) + 1e-6) * ikw.float()
    kk = _rope_ref(kk, posT, cs)
    kq = icache.view(-1, 128)[slots.long()].view(torch.float8_e4m3fn).float()
    torch.testing.assert_close(kq, kk.clamp(-448, 448).to(torch.float8_e4m3fn).float(), rtol=0, atol=0)

    # one query per sequence (its last position), 8 indexer heads, top-64
    Hi, K, H = 8, 64, 16
    Tq = len(ctxs)
    tok_seq = i32(list(range(Tq)))
    tok_ctx = i32(ctxs)
    qi = torch.randn(Tq, Hi, 128).bfloat16().cuda()
    wi = torch.rand(Tq, Hi).cuda()
    maxc = max(ctxs)
    scores = torch.empty(Tq, maxc, device="cuda")
    o.indexer_score(qi, wi, icache, bt, tok_seq, tok_ctx, maxc, scores)
    sel = torch.empty(Tq, K, dtype=torch.int32, device="cuda")
    cnt = torch.empty(Tq, dtype=torch.int32, device="cuda")
    o.topk_select(scores, tok_ctx, K, sel, cnt)
    _check()
    for s, cx in enumerate(ctxs):
        rows = torch.tensor([int(bt[s, p // 64]) * 64 + p % 64 for p in range(cx)], device="cuda")
        kf = icache.view(-1, 128)[rows].view(torch.float8_e4m3fn).float()
        ref = (wi[s][:, None] * torch.relu(qi[s].float() @ kf.t())).sum(0)
        torch.testing.assert_close(scores[s, :cx], ref, rtol=1e-4, atol=1e-4)
        n = min(K, cx)
        assert int(cnt[s]) == n
        got_sel = sel[s, :n].cpu().tolist()
        assert got_sel == sorted(got_sel)
        exp = sorted(torch.topk(scores[s, :cx], n).indices.cpu().tolist())
        assert got_sel == exp

    # sparse MLA over the selected rows
    q = torch.randn(Tq, H, 576).bfloat16().cuda()
    scale = 1 / math.sqrt(192)
    nsplit = 3
    po = torch.empty(Tq * H, nsplit, 512, device="cuda")
    pml = torch.empty(Tq * H, nsplit, 2, device="cuda")
    out = torch.empty(Tq, H, 512, dtype=torch.bfloat16, device="cuda")
    o.sparse_mla_decode(q, lat, bt, tok_seq, sel, cnt, scale, po, pml, out)
    _check()
    for s in range(Tq):
        n = int(cnt[s])
        pos_sel = sel[s, :n].long()
        rows = torch.tensor([int(bt[s, int(p) // 64]) * 64 + int(p) % 64 for p in pos_sel], device="cuda")
        R = lat.view(-1, 576)[rows].float()
        logit = (q[s].float() @ R.t()) * scale
        ref = torch.softmax(logit, -1) @ R[:, :512]
        torch.testing.assert_close(out[s].float(), ref, rtol=2e-2, atol=2e-2)


def test_head_gemv_and_rope_heads():
    T, H, K, N = 5, 6, 512, 128
    x = torch.randn(T, H, K).bfloat16().cuda()
    W = (torch.randn(H, N, K) * 0.05).bfloat16().cuda()
    out = torch.empty(T, H, N, dtype=torch.bfloat16, device="cuda")
    _ops().head_gemv(x, W, out)
    _check()
    ref = torch.einsum("thk,hnk->thn", x.float(), W.float())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    _, _, cs = _setup([40])
    y = torch.randn(T, H, 192).bfloat16().cuda()
    pos = torch.tensor([0, 3, 7, 20, 39], dtype=torch.int32, device="cuda")
    ref = _rope_ref(y[..., 128:].float(), pos.long()[:, None], cs)
    _ops().rope_heads(y, H, 128, pos, cs)
    _check()
    torch.testing.assert_close(y[..., 128:].float(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("H", [16, 40, 64])
def test_sparse_mla_tc_matches_reference(H):
    """The tcgen05 sparse MLA (keys on the MMA's M side, heads on N, O^T in TMEM) against fp32 softmax
    attention over the selected latent rows and against the CUDA-core kernel: selections of 0 to 700
    rows (several 128-key tiles, empty splits), head counts that fill one, one and a part, and two
    32-head groups, two calls in a row."""
    o = _ops()
    from r9700_stack_b200.utils import status

    ctxs = [900, 130, 5, 1, 700]
    counts = [700, 130, 5, 0, 257]
    nblk, bt, _ = _setup(ctxs, seed=4)
    g = torch.Generator().manual_seed(7)
    lat = (torch.randn(nblk, 64, 576, generator=g) * 0.5).bfloat16().cuda()
    Tq, K = len(ctxs), 768
    sel = torch.full((Tq, K), -1, dtype=torch.int32)
    for s, (cx, n) in enumerate(zip(ctxs, counts)):
        sel[s, :n] = torch.randperm(cx, generator=g)[:n].sort().values.int()
    sel, cnt = sel.cuda(), torch.tensor(counts, dtype=torch.int32, device="cuda")
    tok_seq = torch.arange(Tq, dtype=torch.int32, device="cuda")
    q = torch.randn(Tq, H, 576, generator=g).bfloat16().cuda()
    scale = 1 / math.sqrt(192)
    nsplit = 4
    po = torch.empty(Tq * H, nsplit, 512, device="cuda")
    pml = torch.empty(Tq * H, nsplit, 2, device="cuda")
    outs = []
    for _ in range(2):
        out = torch.full((Tq, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
        o.sparse_mla_decode_tc(q, lat, bt, tok_seq, sel, cnt, scale, po, pml, out, status.status(torch.device("cuda")))
        _check()
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    simple = torch.empty(Tq, H, 512, dtype=torch.bfloat16, device="cuda")
    o.sparse_mla_decode(q, lat, bt, tok_seq, sel, cnt, scale, po, pml, simple)
    _check()
    for s in range(Tq):
        n = counts[s]
        if n == 0:
            assert torch.all(outs[0][s] == 0)
            continue
        pos = sel[s, :n].long().cpu()
        rows = torch.tensor([int(bt[s, int(p) // 64]) * 64 + int(p) % 64 for p in pos], device="cuda")
        R = lat.view(-1, 576)[rows].float()
        ref = torch.softmax((q[s].float() @ R.t()) * scale, -1) @ R[:, :512]
        err = float((outs[0][s].float() - ref).norm() / ref.norm())
        assert err < 1e-2, (s, err)  # bf16 probabilities in the P V product
        torch.testing.assert_close(outs[0][s].float(), simple[s].float(), rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("Hi", [8, 20, 64])
def test_indexer_score_long_context(Hi):
    """Indexer scores (tcgen05 by default: e4m3 keys widened to bf16, heads on the MMA's N side)
    against w . relu(q k^T) in fp32 over several 128-key tiles, a context that ends mid-tile,
    positions past it (-inf) and a score row longer than every context."""
    o = _ops()
    from r9700_stack_b200.utils import status

    ctxs = [900, 129, 1]
    nblk, bt, _ = _setup(ctxs, seed=2)
    g = torch.Generator().manual_seed(3)
    icache = (torch.randn(nblk, 64, 128, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8).cuda()
    Tq = len(ctxs)
    qi = torch.randn(Tq, Hi, 128, generator=g).bfloat16().cuda()
    wi = torch.rand(Tq, Hi, generator=g).cuda()
    tok_seq = torch.arange(Tq, dtype=torch.int32, device="cuda")
    tok_ctx = torch.tensor(ctxs, dtype=torch.int32, device="cuda")
    maxc = 1024
    scores = torch.full((Tq, maxc + 8), float("nan"), device="cuda")
    o.indexer_score(qi, wi, icache, bt, tok_seq, tok_ctx, maxc, scores, status.status(torch.device("cuda")))
    _check()
    for s, cx in enumerate(ctxs):
        rows = torch.tensor([int(bt[s, p // 64]) * 64 + p % 64 for p in range(cx)], device="cuda")
        kf = icache.view(-1, 128)[rows].view(torch.float8_e4m3fn).float()
        ref = (wi[s][:, None] * torch.relu(qi[s].float() @ kf.t())).sum(0)
        torch.testing.assert_close(scores[s, :cx], ref, rtol=1e-4, atol=1e-3)
        assert torch.all(scores[s, cx:maxc] == float("-inf"))


def test_sparse_mla_tc_pipelined_grid():
    """A grid large enough for the pipelined tcgen05 kernel (40 tokens x 2 head groups x 4 splits >= two
    CTAs per SM): every token against fp32 softmax attention over its selected rows."""
    o = _ops()
    from r9700_stack_b200.utils import status

    Tq, H, K = 40, 64, 640
    ctxs = [700 + 7 * i for i in range(Tq)]
    nblk, bt, _ = _setup(ctxs, seed=6)
    g = torch.Generator().manual_seed(8)
    lat = (torch.randn(nblk, 64, 576, generator=g) * 0.5).bfloat16().cuda()
    counts = [K if i % 5 else 300 + i for i in range(Tq)]
    sel = torch.full((Tq, K), -1, dtype=torch.int32)
    for s in range(Tq):
        sel[s, :counts[s]] = torch.randperm(ctxs[s], generator=g)[:counts[s]].sort().values.int()
    sel, cnt = sel.cuda(), torch.tensor(counts, dtype=torch.int32, device="cuda")
    tok_seq = torch.arange(Tq, dtype=torch.int32, device="cuda")
    q = torch.randn(Tq, H, 576, generator=g).bfloat16().cuda()
    scale = 1 / math.sqrt(192)
    po = torch.empty(Tq * H, 4, 512, device="cuda")
    pml = torch.empty(Tq * H, 4, 2, device="cuda")
    out = torch.full((Tq, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
    o.sparse_mla_decode_tc(q, lat, bt, tok_seq, sel, cnt, scale, po, pml, out, status.status(torch.device("cuda")))
    _check()
    for s in range(Tq):
        n = counts[s]
        pos = sel[s, :n].long().cpu()
        rows = torch.tensor([int(bt[s, int(p) // 64]) * 64 + int(p) % 64 for p in pos], device="cuda")
        R = lat.view(-1, 576)[rows].float()
        ref = torch.softmax((q[s].float() @ R.t()) * scale, -1) @ R[:, :512]
        err = float((out[s].float() - ref).norm() / ref.norm())
        assert err < 1e-2, (s, err)


@pytest.mark.parametrize("N,K", [(512, 128), (128, 512)])
def test_head_project_wide_batch_matches_head_gemv(N, K):
    """Prefill-sized per-head projections (one tcgen05 GEMM per head on strided views) against the
    CUDA-core head_gemv on the same strided operands."""
    from r9700_stack_b200.models.mla_moe import head_project

    T, H = 300, 6
    g = torch.Generator().manual_seed(4)
    xs = torch.randn(T, H, K + 64, generator=g).bfloat16().cuda()  # strided: extra columns per head
    W = (torch.randn(H, N, K, generator=g) * 0.05).bfloat16().cuda()
    a = torch.zeros(T, H, N + 64, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros_like(a)
    head_project(xs[:, :, :K], W, a[:, :, :N])
    _ops().head_gemv(xs[:, :, :K], W, b[:, :, :N])
    _check()
    torch.testing.assert_close(a[:, :, :N].float(), b[:, :, :N].float(), rtol=2e-2, atol=2e-2)
    assert torch.all(a[:, :, N:] == 0)
