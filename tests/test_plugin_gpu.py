"""The vLLM-facing pieces on the GPU, each against a PyTorch fp32 reference: the compressed-tensors
NVFP4 and fp8 schemes after the swap (load-time conversion + forward), the exl3 linear method (GEMV
and wide-batch paths), the CUSTOM attention backend's cache write + paged attention over vLLM-style
metadata, and the fused RMSNorm installed into vLLM's norm modules."""
import pytest
import torch

pytestmark = pytest.mark.gpu
vllm = pytest.importorskip("vllm")


def _cos(a, b):
    return float(torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


def test_nvfp4_scheme_forward():
    from r9700_stack_b200.ops import linear as L
    from r9700_stack_b200.plugin.quant_ct import _Nvfp4Scheme
    from r9700_stack_b200.quant import formats as F

    torch.manual_seed(0)
    N, K, M = 384, 512, 7
    widths = [256, 128]  # a fused layer of two shards, each with its own global scale
    layer = torch.nn.Module()
    packs, scales, gs, ref_rows = [], [], [], []
    for n in widths:
        w = torch.randn(n, K) * 0.02
        p, s16, g = F.quantize_nvfp4(w)
        packs.append(p)
        scales.append(s16)
        gs.append(g)
        ref_rows.append(F.dequant_nvfp4(p, s16, g))
    layer.weight_packed = torch.nn.Parameter(torch.cat(packs).cuda(), requires_grad=False)
    layer.weight_scale = torch.nn.Parameter(torch.cat(scales).cuda().view(torch.float8_e4m3fn), requires_grad=False)
    layer.weight_global_scale = torch.nn.Parameter(torch.tensor(gs).cuda(), requires_grad=False)
    layer.logical_widths = widths
    sch = _Nvfp4Scheme()
    sch.process_weights_after_loading(layer)
    assert not hasattr(layer, "weight_packed")
    x = torch.randn(M, K, device="cuda").bfloat16()
    bias = torch.randn(N, device="cuda").bfloat16()
    y = sch.apply_weights(layer, x.view(1, M, K), bias)
    assert y.shape == (1, M, N)
    ref = x.float().cpu() @ torch.cat(ref_rows).T + bias.float().cpu()
    assert _cos(y.float().cpu().view(M, N), ref) > 0.99


def test_fp8_block_scheme_forward():
    from r9700_stack_b200.plugin.quant_ct import _Fp8Scheme

    torch.manual_seed(1)
    N, K, M = 256, 384, 5
    w = torch.randn(N, K) * 0.05
    s = w.view(2, 128, 3, 128).abs().amax((1, 3)) / 448
    q = (w / s.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(torch.float8_e4m3fn)
    layer = torch.nn.Module()
    layer.weight = torch.nn.Parameter(q.cuda(), requires_grad=False)
    layer.weight_scale = torch.nn.Parameter(s.cuda(), requires_grad=False)
    sch = _Fp8Scheme()
    sch.process_weights_after_loading(layer)
    x = torch.randn(M, K, device="cuda").bfloat16()
    y = sch.apply_weights(layer, x)
    ref = x.float().cpu() @ (q.float() * s.repeat_interleave(128, 0).repeat_interleave(128, 1)).T
    assert _cos(y.float().cpu(), ref) > 0.995


@pytest.mark.parametrize("M", [4, 40])
def test_exl3_linear_method(M):
    from r9700_stack_b200.ops import exl3 as X
    from r9700_stack_b200.plugin.quant_exl3 import Exl3Config, Exl3LinearMethod
    from r9700_stack_b200.quant import exl3 as E

    n_in, n_out, K = 256, 384, 3
    meth = Exl3LinearMethod(Exl3Config(bits=K), K)
    layer = torch.nn.Module()
    meth.create_weights(layer, n_in, [n_out], n_in, n_out, torch.bfloat16)
    src = X.random_linear(n_in, n_out, K, "cuda", seed=5)
    layer.trellis.data.copy_(src.trellis.cpu())
    layer.suh.data.copy_(src.suh.cpu())
    layer.svh.data.copy_(src.svh.cpu())
    for name in ("trellis", "suh", "svh"):
        getattr(layer, name).data = getattr(layer, name).data.cuda()
    meth.process_weights_after_loading(layer)
    x = torch.randn(M, n_in, device="cuda").bfloat16()
    y = meth.apply(layer, x)
    W = E.dequant(src.trellis.cpu(), src.suh.cpu(), src.svh.cpu(), K, E.MCG)  # fp32 [in, out] oracle
    ref = x.float().cpu() @ W
    assert _cos(y.float().cpu(), ref) > 0.995


def test_custom_backend_cache_and_attention():
    """kv_cache_write + paged_attention over vLLM-style metadata (query start locations, full sequence
    lengths, block table) against causal SDPA on the e4m3-rounded keys and values."""
    from r9700_stack_b200 import _native
    from r9700_stack_b200.plugin.attention import token_layout

    torch.manual_seed(2)
    D, Hq, Hkv, blk = 128, 8, 2, 64
    seqs = [(70, 70), (130, 3), (40, 1)]  # (total length, new tokens this step)
    nb = 16
    kc = torch.zeros(nb, Hkv, blk, D, dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    table = torch.zeros(len(seqs), 4, dtype=torch.int32, device="cuda")
    nxt, allk, allv = 1, [], []
    for i, (L_, _) in enumerate(seqs):
        for j in range(-(-L_ // blk)):
            table[i, j] = nxt
            nxt += 1
        k = torch.randn(L_, Hkv, D, device="cuda").bfloat16()
        v = torch.randn(L_, Hkv, D, device="cuda").bfloat16()
        slots = torch.tensor([int(table[i, t // blk]) * blk + t % blk for t in range(L_)], device="cuda")
        _native.ops().kv_cache_write(k, v, slots, kc, vc, 1.0, 1.0)
        allk.append(k)
        allv.append(v)
    T = sum(n for _, n in seqs)
    q = torch.randn(T, Hq, D, device="cuda").bfloat16()
    qsl = torch.tensor([0] + list(torch.cumsum(torch.tensor([n for _, n in seqs]), 0)), dtype=torch.int32,
                       device="cuda")
    seq_lens = torch.tensor([L_ for L_, _ in seqs], dtype=torch.int32, device="cuda")
    seq, ctx = token_layout(qsl, seq_lens, T)
    out = torch.empty(T, Hq * D, dtype=torch.bfloat16, device="cuda")
    scale = D ** -0.5
    _native.ops().paged_attention(q, kc, vc, table, seq, ctx, scale, 1.0, 1.0, None, out, None, None, 0)
    torch.cuda.synchronize()
    r0 = 0
    for i, (L_, n) in enumerate(seqs):
        k8 = allk[i].float().to(torch.float8_e4m3fn).float()
        v8 = allv[i].float().to(torch.float8_e4m3fn).float()
        for t in range(n):
            pos = L_ - n + t
            qt = q[r0 + t].float().view(Hkv, Hq // Hkv, D)
            s = torch.einsum("hgd,lhd->hgl", qt, k8[: pos + 1]) * scale
            o = torch.einsum("hgl,lhd->hgd", s.softmax(-1), v8[: pos + 1]).reshape(Hq * D)
            assert _cos(out[r0 + t].float(), o) > 0.999, (i, t)
        r0 += n


def test_installed_rmsnorm_matches_vllm():
    from vllm.config import VllmConfig, set_current_vllm_config
    from vllm.model_executor.layers.layernorm import GemmaRMSNorm, RMSNorm

    from r9700_stack_b200.plugin.models import install

    with set_current_vllm_config(VllmConfig()):
        for cls in (RMSNorm, GemmaRMSNorm):
            m = cls(512, eps=1e-6).cuda()
            m.weight.data.copy_(torch.randn(512) * 0.1 + (0.0 if cls is GemmaRMSNorm else 1.0))
            x = torch.randn(9, 512, device="cuda").bfloat16()
            r = torch.randn(9, 512, device="cuda").bfloat16()
            want, want_r = m.forward_native(x.clone(), r.clone())
            assert install(m) == 1
            got, got_r = m(x.clone(), r.clone())
            torch.testing.assert_close(got_r, want_r)
            torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
