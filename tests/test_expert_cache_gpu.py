"""Host-resident experts behind the device LRU: same tokens as fully resident experts, hit / miss
accounting, deterministic victims, and the kernel-level LRU state against a Python model."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_lru_route_matches_python_model():
    from r9700_stack_b200.ops import linear as L
    from r9700_stack_b200.ops.expert_cache import ExpertCache

    E, S, H, I = 12, 5, 256, 256
    mk = lambda n, k: L.stack_experts([L.mx_from_float((torch.randn(n, k) * 0.05).cuda(), search=False) for _ in range(E)])
    c = ExpertCache(mk(I, H), mk(I, H), mk(H, I), E, S, "cuda")
    resident, stamp, now = {}, {}, 0  # python model: slot -> expert, slot -> stamp
    steps = [[1, 2, 3], [3, 4, 5], [6, 1, 2], [7, 8, 9], [1, 9, 10], [11, 0, 3]]
    for ids in steps:
        now += 1
        need = sorted(set(ids))
        for s, e in resident.items():
            if e in need:
                stamp[s] = now
        miss = [e for e in need if e not in resident.values()]
        cands = sorted([s for s in range(S) if s not in resident] + [s for s in resident if resident[s] not in need],
                       key=lambda s: (stamp.get(s, -1) if s in resident else -1, s))
        for e, v in zip(miss, cands):
            resident[v] = e
            stamp[v] = now
        t = torch.tensor(ids, dtype=torch.int32, device="cuda").view(1, -1)
        slot_ids = torch.zeros_like(t)
        c.route(t, 0, slot_ids)
        torch.cuda.synchronize()
        inv = {e: s for s, e in resident.items()}
        assert slot_ids.view(-1).tolist() == [inv[e] for e in ids]
        assert c.expert_of.tolist() == [resident.get(s, -1) for s in range(S)]
    # the slot arrays hold the experts they are mapped to
    g0 = c.weights[0]
    for s, e in resident.items():
        qb = c.bytes[0]
        assert torch.equal(c.dev[0][s * qb:(s + 1) * qb].cpu(), c.host[0][e * qb:(e + 1) * qb])
    st = c.stats()
    assert st["hits"] + st["misses"] == sum(len(set(x)) for x in steps)


def test_moe_model_with_cache_matches_resident():
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_moe
    from r9700_stack_b200.utils import status

    cfg = tiny_moe()
    prompts = [[5, 6, 7, 8, 9, 10], [40, 41, 42]]
    outs = []
    for cached in (False, True):
        ec = EngineConfig(max_batch=2, max_model_len=128, max_prefill_tokens=64, cuda_graphs=cached,
                          graph_batch_sizes=[1, 2])
        from r9700_stack_b200.engine.llm import build_model
        from r9700_stack_b200.models.config import ParallelConfig

        m = build_model(cfg, ParallelConfig(), torch.device("cuda"), seed=9)
        if cached:
            m.enable_expert_cache(slots=6)  # < 8 experts, >= the experts one decode step can route to
        llm = LLM(cfg, ec, seed=9, model=m)
        outs.append(llm.generate(prompts, SamplingParams(max_tokens=8)))
        torch.cuda.synchronize()
        status.check()
        if cached:
            st = m.caches[0].stats()
            assert st["misses"] > 0 and st["hits"] > 0
    assert outs[0] == outs[1]


def test_routing_profile_warm_start(tmp_path):
    """A routing profile recorded while serving preloads each layer's most routed experts: the warm
    cache misses less on the same traffic and the tokens stay those of resident experts."""
    from r9700_stack_b200.engine.llm import LLM, build_model
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, ParallelConfig, tiny_moe
    from r9700_stack_b200.ops.expert_cache import RoutingProfile

    cfg = tiny_moe()
    prompts = [[5, 6, 7, 8, 9, 10], [40, 41, 42]]
    ec = EngineConfig(max_batch=2, max_model_len=128, max_prefill_tokens=64, cuda_graphs=False)
    m = build_model(cfg, ParallelConfig(), torch.device("cuda"), seed=9)
    m.record_routing(True)
    want = LLM(cfg, ec, seed=9, model=m).generate(prompts, SamplingParams(max_tokens=8))
    path = str(tmp_path / "expertprofile.safetensors")
    m.routing_profile.save(path)
    prof = RoutingProfile.load(path)
    assert int(prof.counts.sum()) == int(m.routing_profile.counts.sum().cpu()) > 0
    misses = {}
    for warm in (False, True):
        mm = build_model(cfg, ParallelConfig(), torch.device("cuda"), seed=9)
        mm.enable_expert_cache(slots=6, profile=path if warm else None)
        if warm:
            top = prof.top(0, 6)
            assert sorted(int(e) for e in mm.caches[0].expert_of.tolist()) == sorted(top)
        got = LLM(cfg, ec, seed=9, model=mm).generate(prompts, SamplingParams(max_tokens=8))
        assert got == want
        misses[warm] = sum(c.stats()["misses"] for c in mm.caches)
    assert misses[True] < misses[False], misses
