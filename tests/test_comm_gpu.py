"""Fused all-reduce path on one GPU (world size 1: the producer pushes to its own region and the
consumer reduces one slot; producer and consumer run in stream order, so no kernel waits on another
that could be co-scheduled)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _check():
    from r9700_stack_b200.utils import status

    torch.cuda.synchronize()
    status.check()


@pytest.mark.parametrize("mode", ["push", "pull", "ll"])
def test_fused_allreduce_norm_matches_unfused(mode, monkeypatch):
    from r9700_stack_b200 import knobs
    from r9700_stack_b200.ops import linear as L
    from r9700_stack_b200.parallel.symm import SymmComm

    monkeypatch.setenv("R9K_AR_MODE", mode)
    knobs.refresh()

    torch.manual_seed(0)
    H, K, T = 1024, 2048, 12
    comm = SymmComm(H, max_tokens=16, calls_per_step=2, device="cuda")
    w = L.mx_from_float((torch.randn(H, K) * 0.02).cuda(), tiled=True)
    x = L.quant_act(torch.randn(T, K).bfloat16().cuda())
    nw = (torch.randn(H) * 0.1).bfloat16().cuda()
    resid = torch.randn(T, H).bfloat16().cuda()
    # unfused reference: GEMM -> bf16 y; add + norm + quant
    y = L.mx_linear(x, w)
    r1 = resid.clone()
    a1 = L.alloc_act(T, H, "cuda")
    L.rmsnorm(y, nw, 1e-6, plus_one=True, residual=r1, residual_out=r1, quant_out=a1)
    # fused: push epilogue + reduce-norm, two steps so both buffers and epochs are exercised
    for step in range(3):
        r2 = resid.clone()
        a2 = L.alloc_act(T, H, "cuda")
        comm.step_begin()
        if mode in ("push", "ll"):
            comm.gemm_push(x, w, call=0)
        else:
            L.mx_linear(x, w, out=comm.out_buffer(0, T))
        comm.ar_rmsnorm(0, T, nw, 1e-6, True, residual=r2, residual_out=r2, quant_out=a2)
        if mode in ("push", "ll"):
            comm.push(y, call=1)
        else:
            comm.out_buffer(1, T).copy_(y)
        y3 = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        r3 = resid.clone()
        comm.ar_rmsnorm(1, T, nw, 1e-6, True, residual=r3, residual_out=r3, y=y3)
        _check()
        assert torch.equal(r1, r2) and torch.equal(a1.q, a2.q), step
        assert torch.equal(r1, r3)
    comm.close()
    knobs.refresh()


def test_tiny_model_fused_comm_equals_plain():
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_hybrid
    from r9700_stack_b200.parallel.symm import SymmComm

    cfg = tiny_hybrid()
    prompts = [list(range(3, 40)), list(range(100, 117))]
    outs = []
    for fused in (False, True):
        comm = SymmComm(cfg.hidden, max_tokens=4, calls_per_step=2 * cfg.layers, device="cuda") if fused else None
        ec = EngineConfig(max_batch=4, max_model_len=256, max_prefill_tokens=128, graph_batch_sizes=[1, 2, 4])
        llm = LLM(cfg, ec, seed=5, comm=comm)
        outs.append(llm.generate(prompts, SamplingParams(max_tokens=6)))
        _check()
        del llm
        if comm is not None:
            comm.close()
    assert outs[0] == outs[1]


def test_ll_wait_runs_out_and_reports(monkeypatch):
    """A consumer whose data never arrives gives up after its limit, records kErrPeerTimeout in the
    status word and returns; the context stays usable (the next call on the same stream works)."""
    from r9700_stack_b200 import knobs
    from r9700_stack_b200.ops import linear as L
    from r9700_stack_b200.parallel.symm import SymmComm
    from r9700_stack_b200.utils import status

    monkeypatch.setenv("R9K_AR_MODE", "ll")
    knobs.refresh()
    H, T = 1024, 4
    comm = SymmComm(H, max_tokens=T, calls_per_step=2, device="cuda", timeout_s=0.001)
    nw = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    a = L.alloc_act(T, H, "cuda")
    st = status.status(torch.device("cuda"))
    comm.step_begin()
    comm.ar_rmsnorm(0, T, nw, 1e-6, False, quant_out=a)  # nothing was pushed for call 0 of this step
    torch.cuda.synchronize()
    word = st.tolist()
    assert word[0] == 2 and word[1] == 320, word  # kErrPeerTimeout from the LL consumer
    st.zero_()
    # the same communicator keeps working: push, then reduce
    x = torch.randn(T, H, device="cuda").bfloat16()
    comm.push(x, call=1)
    y = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    comm.ar_rmsnorm(1, T, nw, 1e-6, False, y=y)
    _check()
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
    comm.close()
    knobs.refresh()
