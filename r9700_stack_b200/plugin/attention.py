"""vLLM attention backend ``CUSTOM`` on this library's paged fp8 attention kernels.

Selected with ``--attention-backend CUSTOM`` once ``register()`` ran. The KV cache uses this library's
layout -- per layer ``[2, blocks, kv_heads, 64, head_dim]`` e4m3 bytes, so ``kv_cache[0]`` and
``kv_cache[1]`` are exactly the ``[blocks, kv_heads, 64, head_dim]`` K / V pools the kernels read --
and vLLM's FlashAttention metadata builder (query start locations, sequence lengths, block table).
Per layer: ``do_kv_cache_update`` stores the step's keys and values (``kv_cache_write``: e4m3 with
the layer's scales, by slot), ``forward`` derives each token's sequence and causal context length from
the metadata and runs ``paged_attention`` (bf16 queries, GQA, head 128 or 256).
Reference: r9700_vllm/attn/triton3d.py:260-290 (backend CUSTOM over the reference's paged kernels).
"""
from __future__ import annotations

import torch
from vllm.v1.attention.backends.flash_attn import (
    FlashAttentionBackend,
    FlashAttentionImpl,
    FlashAttentionMetadataBuilder,
)

from .. import _native

KV_BLOCK = 64


def token_layout(query_start_loc: torch.Tensor, seq_lens: torch.Tensor, T: int):
    """(sequence index, causal context length) of every token of a batch laid out by query start
    locations [S + 1] with full sequence lengths [S] (new tokens last). No host synchronisation."""
    S = seq_lens.shape[0]
    q_lens = query_start_loc[1:] - query_start_loc[:-1]
    seq = torch.repeat_interleave(torch.arange(S, device=seq_lens.device, dtype=torch.int32), q_lens, output_size=T)
    pos_in_q = torch.arange(T, device=seq_lens.device, dtype=torch.int32) - query_start_loc[:-1][seq].int()
    ctx = (seq_lens[seq] - q_lens[seq]).int() + pos_in_q + 1
    return seq, ctx


class R9kAttentionImpl(FlashAttentionImpl):
    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping) -> None:
        k_cache, v_cache = _pools(kv_cache)
        n = slot_mapping.shape[0]
        _native.ops().kv_cache_write(key[:n], value[:n], slot_mapping.long(), k_cache, v_cache,
                                     float(layer._k_scale_float), float(layer._v_scale_float))

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("R9kAttentionImpl: fused output quantisation")
        if attn_metadata is None:  # profiling run
            return output.fill_(0)
        T = attn_metadata.num_actual_tokens
        k_cache, v_cache = _pools(kv_cache)
        seq, ctx = token_layout(attn_metadata.query_start_loc, attn_metadata.seq_lens, T)
        out = output[:T].view(T, -1)
        _native.ops().paged_attention(query[:T].contiguous(), k_cache, v_cache, attn_metadata.block_table.int(),
                                      seq, ctx, float(self.scale), float(layer._k_scale_float),
                                      float(layer._v_scale_float), None, out, None, None, 0)
        return output


def _pools(kv_cache: torch.Tensor):
    kc, vc = kv_cache.unbind(0)
    return kc.view(torch.uint8), vc.view(torch.uint8)


class R9kAttentionBackend(FlashAttentionBackend):
    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls():
        return R9kAttentionImpl

    @staticmethod
    def get_builder_cls():
        return FlashAttentionMetadataBuilder

    @staticmethod
    def get_supported_kernel_block_sizes():
        return [KV_BLOCK]

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        if block_size != KV_BLOCK:
            raise ValueError(f"R9kAttentionBackend: KV block size must be {KV_BLOCK}")
        return (2, num_blocks, num_kv_heads, block_size, head_size)

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension: bool = False) -> tuple[int, ...]:
        if include_num_layers_dimension:
            return (1, 0, 2, 3, 4, 5)
        return (0, 1, 2, 3, 4)

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size in (128, 256)

    @classmethod
    def supports_kv_cache_dtype(cls, kv_cache_dtype) -> bool:
        return kv_cache_dtype is not None and str(kv_cache_dtype).startswith("fp8")

    @classmethod
    def supports_sink(cls) -> bool:
        return False

    @classmethod
    def supports_compute_capability(cls, capability) -> bool:
        return getattr(capability, "major", 0) == 10
