"""The vLLM integration points against the installed vLLM, on a host without a GPU: what
``register()`` registers (quantization configs, model archs, the CUSTOM attention backend), the
platform and communicator classes, the scheme swap of the compressed-tensors override and the
exl3 config parsing. Reference counterpart: tests/test_integration.py (entry points, platform class,
communicator subclass, registry overrides)."""
import os

import pytest
import torch

vllm = pytest.importorskip("vllm")


@pytest.fixture(scope="module")
def registered():
    from r9700_stack_b200 import plugin

    return plugin.register()


def test_register_lists_every_piece(registered):
    kinds = {x.split(":")[0] for x in registered}
    assert {"ops", "quant", "models", "attn"} <= kinds, registered
    from r9700_stack_b200 import plugin

    assert plugin.register() is registered  # idempotent


def test_quant_configs_registered(registered):
    from vllm.model_executor.layers.quantization import get_quantization_config

    from r9700_stack_b200.plugin.quant_ct import R9kCompressedTensorsConfig
    from r9700_stack_b200.plugin.quant_exl3 import Exl3Config

    assert get_quantization_config("compressed-tensors") is R9kCompressedTensorsConfig
    assert get_quantization_config("exl3") is Exl3Config
    cfg = Exl3Config.from_config({"bits": 3, "codebook": "mul1", "bits_overrides": {"mlp.down_proj": 4}})
    assert cfg.get_name() == "exl3" and cfg.codebook == "mul1"
    assert cfg.bits_for("model.layers.3.mlp.down_proj") == 4 and cfg.bits_for("model.layers.3.self_attn.o_proj") == 3
    with pytest.raises(ValueError):
        Exl3Config(bits=9)


def test_model_archs_registered(registered):
    from vllm import ModelRegistry

    from r9700_stack_b200.plugin.models import ARCHS

    archs = set(ModelRegistry.get_supported_archs())
    for arch, qual in ARCHS.items():
        assert arch in archs
        info = ModelRegistry.models[arch]
        assert f"{info.module_name}:{info.class_name}" == qual, (arch, info)


def test_attention_backend_registered(registered):
    from vllm.v1.attention.backends import registry as R

    assert R._ATTN_OVERRIDES[R.AttentionBackendEnum.CUSTOM] == "r9700_stack_b200.plugin.attention.R9kAttentionBackend"


def test_scheme_swap_is_per_instance():
    from vllm.model_executor.layers.quantization.compressed_tensors.schemes import CompressedTensorsW4A4Fp4

    from r9700_stack_b200.plugin.quant_ct import _Nvfp4Scheme, served_scheme

    try:
        a, b = CompressedTensorsW4A4Fp4(), CompressedTensorsW4A4Fp4()
    except Exception as e:  # the stock constructor may probe a GPU kernel backend
        pytest.skip(f"stock NVFP4 scheme needs a GPU here: {type(e).__name__}")
    served_scheme(a)
    assert isinstance(a, _Nvfp4Scheme) and isinstance(a, CompressedTensorsW4A4Fp4)
    assert type(b) is CompressedTensorsW4A4Fp4  # the stock class itself is untouched
    assert served_scheme(None) is None


def test_token_layout():
    from r9700_stack_b200.plugin.attention import token_layout

    qsl = torch.tensor([0, 3, 4, 9], dtype=torch.int32)  # query lengths 3, 1, 5
    seq_lens = torch.tensor([10, 7, 5], dtype=torch.int32)  # context incl. the new tokens
    seq, ctx = token_layout(qsl, seq_lens, 9)
    assert seq.tolist() == [0, 0, 0, 1, 2, 2, 2, 2, 2]
    assert ctx.tolist() == [8, 9, 10, 7, 1, 2, 3, 4, 5]


def test_install_rebinds_norms():
    from vllm.model_executor.layers.layernorm import GemmaRMSNorm, RMSNorm

    from r9700_stack_b200.plugin.models import install

    from vllm.config import VllmConfig, set_current_vllm_config

    try:
        vc = VllmConfig()
    except RuntimeError as e:  # vLLM cannot infer a device type on a host without a GPU
        pytest.skip(f"VllmConfig needs a device here: {e}")
    with set_current_vllm_config(vc):  # vLLM custom-op modules are built under a config
        m = torch.nn.Sequential(RMSNorm(256), GemmaRMSNorm(256), torch.nn.Linear(4, 4))
    assert install(m) == 2 and install(m) == 0
    x = torch.randn(3, 256)  # fp32: the kernel takes bf16 only, so vLLM's own forward runs
    assert m[0]._r9k_plus_one is False and m[1]._r9k_plus_one is True
    with set_current_vllm_config(vc):
        torch.testing.assert_close(m[0](x), m[0]._r9k_stock_forward(x))


def test_platform_and_communicator_classes():
    from r9700_stack_b200.plugin import platform

    assert platform.detect() is None  # no B200 here
    try:
        cls = platform.B200Platform
    except Exception as e:
        pytest.skip(f"vLLM's CUDA platform needs a driver: {type(e).__name__}")
    assert cls.get_device_communicator_cls() == "r9700_stack_b200.plugin.communicator.R9kCommunicator"
    from vllm.distributed.device_communicators.cuda_communicator import CudaCommunicator

    from r9700_stack_b200.plugin.communicator import R9kCommunicator

    assert issubclass(R9kCommunicator, CudaCommunicator)


def test_disable_opt_out(monkeypatch):
    import importlib

    from r9700_stack_b200 import knobs

    monkeypatch.setenv("R9K_DISABLE", "plugin")
    knobs.refresh()
    import r9700_stack_b200.plugin as P

    saved = P._registered
    P._registered = None
    try:
        assert P.register() == []
    finally:
        P._registered = saved
        monkeypatch.delenv("R9K_DISABLE")
        knobs.refresh()
