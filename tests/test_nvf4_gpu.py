"""Native NVFP4 GEMM (R9K_NVFP4=native): the checkpoint's e2m1 codes and e4m3 block-16 scales served
unconverted, against the fp32 dequantisation of the same NVFP4 tensor (the products are exact in bf16,
so the only rounding is the bf16 activations' and the fp32 accumulation's), and the hybrid model with
native NVFP4 weights against its fp32 oracle."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cos(a, b):
    return float(torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


@pytest.mark.parametrize("N,K,M", [(256, 512, 1), (512, 1024, 16), (1024, 2048, 7), (384, 4096, 40), (256, 512, 200)])
def test_gemm_nvf4_matches_dequant(N, K, M):
    from r9700_stack_b200.ops import linear as L
    from r9700_stack_b200.utils import status

    torch.manual_seed(N + M)
    w = torch.randn(N, K, device="cuda") * 0.02
    packed, s16, g = L.nvfp4_quantize(w)
    nw = L.NVF4Weight.from_checkpoint(packed, s16, g)
    wd = nw.dequant()
    x = torch.randn(M, K, device="cuda").bfloat16()
    y = L.nvf4_linear(x, nw)
    torch.cuda.synchronize()
    status.check()
    ref = x.float() @ wd.T
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=2e-3 * float(ref.abs().max()))


@pytest.mark.parametrize("M", [4, 33])
def test_gemm_nvf4_swiglu(M):
    from r9700_stack_b200.ops import linear as L

    torch.manual_seed(M)
    N, K = 512, 1024
    wg, wu = (L.NVF4Weight.from_checkpoint(*L.nvfp4_quantize(torch.randn(N, K, device="cuda") * 0.03)) for _ in range(2))
    x = torch.randn(M, K, device="cuda").bfloat16()
    y = L.nvf4_swiglu(x, wg, wu)
    g, u = x.float() @ wg.dequant().T, x.float() @ wu.dequant().T
    ref = torch.nn.functional.silu(g) * u
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-3 * float(ref.abs().max()))


def test_hybrid_native_nvfp4_matches_reference(monkeypatch):
    from r9700_stack_b200 import knobs
    from r9700_stack_b200.engine.llm import LLM
    from r9700_stack_b200.engine.scheduler import SamplingParams
    from r9700_stack_b200.models.config import EngineConfig, tiny_hybrid
    from r9700_stack_b200.models.reference import ReferenceState, reference_forward
    from r9700_stack_b200.ops import linear as L

    monkeypatch.setenv("R9K_NVFP4", "native")
    knobs.refresh()
    try:
        cfg = tiny_hybrid(weight_format="nvfp4", lm_head_format="block_fp8", gdn_state_dtype="fp32")
        ec = EngineConfig(max_batch=2, max_model_len=512, max_prefill_tokens=256, cuda_graphs=True,
                          graph_batch_sizes=[1, 2])
        llm = LLM(cfg, ec, seed=3)
        assert isinstance(llm.model.layers[0]["w_in"], L.NVF4Weight) and not llm.model.mx
        prompt = torch.randint(0, cfg.vocab, (70,), generator=torch.Generator().manual_seed(5)).tolist()
        seq = llm.add_request(prompt, SamplingParams(max_tokens=4))
        st = ReferenceState(llm.model)
        llm.step()
        ref = reference_forward(llm.model, prompt, st)[-1]
        assert _cos(llm.runner.ws.logits[0], ref) > 0.999
        for _ in range(3):
            llm.step()
            ref = reference_forward(llm.model, [seq.output[-2]], st)[-1]
            assert _cos(llm.runner.ws.logits[0], ref) > 0.998
    finally:
        monkeypatch.delenv("R9K_NVFP4")
        knobs.refresh()
