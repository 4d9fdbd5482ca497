"""Model configurations.

The synthetic configs mirror the five BASELINE configurations (class-level shapes of the
reference's served models; the reference serves Qwen3.8-27B, Qwen3.8-Flash-Next, GLM-5.3-Flash and
DeepSeek-V4.1-Flash checkpoints: r9700_vllm/models/*.py). Shapes are generic; tests use tiny
variants of the same classes.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace


@dataclass
class HybridConfig:
    """Hybrid Gated-DeltaNet / full-attention decoder (dense SwiGLU FFN or routed MoE FFN)."""

    name: str = "hybrid"
    hidden: int = 5120
    layers: int = 64
    full_attn_interval: int = 4  # every 4th layer is full attention (3:1 GDN:attention)
    vocab: int = 248320
    # full attention
    n_q_heads: int = 24
    n_kv_heads: int = 4
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 10_000_000.0
    attn_output_gate: bool = True
    # gated deltanet
    gdn_k_heads: int = 16
    gdn_v_heads: int = 48
    gdn_head_dim: int = 128
    conv_width: int = 4
    # dense FFN
    ffn: int = 17408
    # MoE FFN (moe_experts == 0 -> dense)
    moe_experts: int = 0
    moe_topk: int = 0
    moe_ffn: int = 0
    moe_shared_ffn: int = 0
    moe_router: str = "softmax"  # softmax | sigmoid
    # numerics / formats
    rms_eps: float = 1e-6
    norm_plus_one: bool = True  # Gemma-style (1 + w) RMSNorm weights
    weight_format: str = "nvfp4"  # nvfp4 (converted to MXFP4 at load) | mxfp8 | bf16
    lm_head_format: str = "block_fp8"  # block_fp8 (converted to MXFP8) | mxfp4 | bf16
    kv_cache_dtype: str = "fp8"
    gdn_state_dtype: str = "bf16"  # bf16 | fp32
    # per-layer int6 embeddings in pinned host memory (Flash-Next class)
    ple_dim: int = 0
    # QSA sparse attention on the full-attention layers (Flash-Next class): top-k 4-token groups by an
    # indexer of qsa_heads x 128 query heads against mean-pooled group keys (0 = dense attention)
    qsa_topk: int = 0
    qsa_heads: int = 4
    # hyper-connections: HC residual streams, sigmoid-gated mix into every block (0 = plain residual)
    hc_streams: int = 0
    init_std: float = 0.02
    tie_embeddings: bool = False
    # speculative decoding
    mtp_layers: int = 0
    drafter: str = ""  # "" | "block" | "mtp"
    draft_block: int = 8

    def is_attention(self, i: int) -> bool:
        return (i + 1) % self.full_attn_interval == 0

    @property
    def attn_layers(self) -> list[int]:
        return [i for i in range(self.layers) if self.is_attention(i)]

    @property
    def gdn_layers(self) -> list[int]:
        return [i for i in range(self.layers) if not self.is_attention(i)]

    def scaled(self, **kw) -> "HybridConfig":
        return replace(self, **kw)


def qwen27b_hybrid() -> HybridConfig:
    """dense hybrid GDN/attention 27B-class."""
    return HybridConfig(name="hybrid-dense-27b", drafter="block", draft_block=8)


def flashnext_moe() -> HybridConfig:
    """hybrid MoE, Flash-Next class (288 experts, top-10)."""
    return HybridConfig(
        name="hybrid-moe-flashnext",
        hidden=2048,
        layers=48,
        n_q_heads=16,
        n_kv_heads=2,
        head_dim=256,
        gdn_k_heads=16,
        gdn_v_heads=32,
        ffn=0,
        moe_experts=288,
        moe_topk=10,
        moe_ffn=512,
        moe_shared_ffn=512,
        weight_format="bf16",
        lm_head_format="bf16",
        ple_dim=256,
        qsa_topk=512,
        hc_streams=4,
        mtp_layers=3,
        drafter="mtp",
    )


def tiny_moe(**kw) -> HybridConfig:
    """A small Flash-Next-class MoE config (bf16 attention/dense, NVFP4 experts), for tests."""
    base = dict(
        name="tiny-moe",
        hidden=256,
        layers=4,
        vocab=512,
        n_q_heads=4,
        n_kv_heads=2,
        head_dim=256,
        gdn_k_heads=2,
        gdn_v_heads=4,
        ffn=0,
        moe_experts=8,
        moe_topk=3,
        moe_ffn=256,
        moe_shared_ffn=256,
        weight_format="bf16",
        lm_head_format="bf16",
    )
    base.update(kw)
    return HybridConfig(**base)


def tiny_hybrid(**kw) -> HybridConfig:
    """A small config of the same class, for tests."""
    base = dict(
        name="tiny-hybrid",
        hidden=256,
        layers=4,
        vocab=512,
        n_q_heads=4,
        n_kv_heads=2,
        head_dim=256,
        rotary_dim=64,
        gdn_k_heads=2,
        gdn_v_heads=4,
        gdn_head_dim=128,
        ffn=512,
        lm_head_format="block_fp8",
    )
    base.update(kw)
    return HybridConfig(**base)


def _glm():
    from .mla_moe import glm53_flash

    return glm53_flash()


def _tiny_mla():
    from .mla_moe import tiny_mla

    return tiny_mla()


def _dsv4():
    from .dsv4 import dsv41_flash

    return dsv41_flash()


def _tiny_dsv4():
    from .dsv4 import tiny_dsv4

    return tiny_dsv4()


MODELS = {
    "dense27b": qwen27b_hybrid,
    "flashnext": flashnext_moe,
    "glm53": _glm,
    "dsv41": _dsv4,
    "tiny-hybrid": tiny_hybrid,
    "tiny-moe": tiny_moe,
    "tiny-mla": _tiny_mla,
    "tiny-dsv4": _tiny_dsv4,
}


def model_config(name: str) -> HybridConfig:
    """A named model preset (the synthetic configs of the BASELINE classes, and their tiny variants)."""
    try:
        return MODELS[name]()
    except KeyError:
        raise ValueError(f"unknown model {name!r}; known: {sorted(MODELS)}") from None


@dataclass
class ParallelConfig:
    tp_size: int = 1
    tp_rank: int = 0
    ep_size: int = 1
    ep_rank: int = 0


@dataclass
class EngineConfig:
    max_batch: int = 16
    max_model_len: int = 32768
    max_prefill_tokens: int = 8192
    kv_block: int = 64
    num_kv_blocks: int = 0  # 0 -> sized from max_batch * max_model_len
    cuda_graphs: bool = True
    graph_batch_sizes: list[int] = field(default_factory=lambda: [1, 2, 4, 8, 16])
    spec_tokens: int = 0  # draft tokens verified per step (0: no speculative decoding)
    spec_method: str = "ngram"  # ngram | mtp | block | dspark
    ep_placement: str = ""  # JSON expert placement (parallel.ep_placement) for MoE models; "" = contiguous
