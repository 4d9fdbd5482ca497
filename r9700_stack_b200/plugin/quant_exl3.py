"""vLLM quantization config "exl3": trellis-coded linears on this library's kernels.

A layer quantised this way stores ``trellis`` (int16 [in/16, out/16, 16 K]), ``suh`` (f16 [in]) and
``svh`` (f16 [out]) -- the tensor set of the EXL3 format (``quant/exl3.py`` defines the decode, the
codebooks and the within-tile order this library uses). Bits per weight K come from the checkpoint's
``quantization_config`` (``bits``, with per-layer ``bits_overrides`` keyed by module prefix);
``codebook`` is ``mcg`` (default) or ``mul1``.

Tensor parallelism: column-parallel layers split the output tiles (``svh`` with them), row-parallel
layers split the input tiles (``suh`` with them); both are 128-aligned so the 128-point Hadamard
rotations stay within a rank (the reference's TP 128-multiple rule, r9700_vllm/quant/exl3.py:9-15).
Forward: at most 16 rows per call run the trellis GEMV (``exl3_gemv`` + ``exl3_finish``), wider
batches dequantise once into a cached bf16 weight for the tcgen05 GEMM.
Reference: r9700_vllm/quant/exl3.py:218-275 (Exl3Config), :295-557 (Exl3LinearMethod).
"""
from __future__ import annotations

from typing import Any

import torch
from torch.nn import Parameter
from vllm.model_executor.layers.linear import LinearBase, LinearMethodBase
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
from vllm.model_executor.utils import set_weight_attrs

from ..ops import exl3 as X
from ..ops import linear as L
from ..quant import exl3 as E


@register_quantization_config("exl3")
class Exl3Config(QuantizationConfig):
    def __init__(self, bits: int = 3, codebook: str = "mcg", bits_overrides: dict[str, int] | None = None):
        super().__init__()
        if not 1 <= int(bits) <= 8:
            raise ValueError(f"exl3: bits per weight must be 1..8, got {bits}")
        if codebook not in ("mcg", "mul1"):
            raise ValueError(f"exl3: codebook must be mcg or mul1, got {codebook!r}")
        self.bits = int(bits)
        self.codebook = codebook
        self.bits_overrides = {k: int(v) for k, v in (bits_overrides or {}).items()}

    def __repr__(self) -> str:
        return f"Exl3Config(bits={self.bits}, codebook={self.codebook})"

    @classmethod
    def get_name(cls) -> str:
        return "exl3"

    @classmethod
    def get_supported_act_dtypes(cls) -> list[torch.dtype]:
        return [torch.bfloat16, torch.float16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # sm_100a kernels

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "Exl3Config":
        return cls(bits=config.get("bits", 3), codebook=config.get("codebook", "mcg"),
                   bits_overrides=config.get("bits_overrides"))

    def bits_for(self, prefix: str) -> int:
        for key, k in self.bits_overrides.items():
            if prefix == key or prefix.endswith("." + key) or prefix.startswith(key + "."):
                return k
        return self.bits

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        if isinstance(layer, LinearBase):
            return Exl3LinearMethod(self, self.bits_for(prefix))
        return None


class Exl3LinearMethod(LinearMethodBase):
    def __init__(self, cfg: Exl3Config, K: int):
        self.cfg = cfg
        self.K = K

    def create_weights(self, layer: torch.nn.Module, input_size_per_partition: int, output_partition_sizes: list[int],
                       input_size: int, output_size: int, params_dtype: torch.dtype, **extra_weight_attrs):
        n_out = sum(output_partition_sizes)
        n_in = input_size_per_partition
        if n_in % 128 or n_out % 128:
            raise ValueError(f"exl3: per-rank shapes must be multiples of 128 (got in={n_in}, out={n_out})")
        trellis = Parameter(torch.empty(n_in // 16, n_out // 16, 16 * self.K, dtype=torch.int16), requires_grad=False)
        set_weight_attrs(trellis, {"input_dim": 0, "output_dim": 1})
        suh = Parameter(torch.empty(n_in, dtype=torch.float16), requires_grad=False)
        set_weight_attrs(suh, {"input_dim": 0})
        svh = Parameter(torch.empty(n_out, dtype=torch.float16), requires_grad=False)
        set_weight_attrs(svh, {"output_dim": 0})
        for name, p in (("trellis", trellis), ("suh", suh), ("svh", svh)):
            set_weight_attrs(p, extra_weight_attrs)
            layer.register_parameter(name, p)
        layer.exl3_K = self.K

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        cb = E.MCG if self.cfg.codebook == "mcg" else E.MUL1
        layer.r9k_exl3 = X.Exl3Linear(layer.trellis.data.contiguous(), layer.suh.data.contiguous(),
                                      layer.svh.data.contiguous(), self.K, cb)
        # bf16 weight for wide batches (M > 16), made now: at load time, outside any graph capture,
        # and finished before a GEMM reads it
        layer.r9k_dense = layer.r9k_exl3.dequant_bf16()

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        w: X.Exl3Linear = layer.r9k_exl3
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        M = x2.shape[0]
        if M <= 16:
            out = torch.empty(M, w.n_out, dtype=torch.bfloat16, device=x.device)
            w.gemv(x2, out)
        else:
            out = L.bf16_linear(x2, layer.r9k_dense)
        if bias is not None:
            out = out + bias
        return out.reshape(*lead, w.n_out).to(x.dtype)
