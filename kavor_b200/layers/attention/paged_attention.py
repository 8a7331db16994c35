"""Paged-KV attention layer (drop-in for kavor/layers/attention/flash_attention_kvcache.py).

``store_kvcache`` and ``Attention`` keep the reference's signatures and
behaviour; the KV write, the varlen/paged prefill attention and the paged
decode attention are the sm_100a kernels of ``libkavor_b200.so``.
"""
from __future__ import annotations

import torch
from torch import nn

from kavor_b200 import _kernels as K
from kavor_b200.utils.context import get_context


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """Write key/value [N, Hkv, hd] rows into the paged cache at slot_mapping
    (flash_attention_kvcache.py:37-46); -1 slots are skipped."""
    K.store_kvcache(key, value, k_cache, v_cache, slot_mapping)


class Attention(nn.Module):
    """flash_attention_kvcache.py:49-84.

    ``k_cache[slot]`` / ``v_cache[slot]`` are [num_blocks, block_size, Hkv, hd]
    views into the page pool, bound by the cache pool. ``forward`` writes the
    step's K/V (unless ``kv_stored``: the fused Qwen3 prologue already wrote
    them) and returns [T, Hq, hd] for prefill or [B, Hq, hd] for decode.
    """

    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int, num_kv_slots: int = 1):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.num_kv_slots = num_kv_slots
        self.k_cache = [torch.tensor([]) for _ in range(num_kv_slots)]
        self.v_cache = [torch.tensor([]) for _ in range(num_kv_slots)]

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, slot: int = 0,
                kv_stored: bool = False) -> torch.Tensor:
        ctx = get_context()
        k_cache, v_cache = self.k_cache[slot], self.v_cache[slot]
        has_cache = k_cache.numel() > 0 and v_cache.numel() > 0
        if has_cache and not kv_stored:
            store_kvcache(k, v, k_cache, v_cache, ctx.slot_mapping)
        if ctx.is_prefill:
            if ctx.block_tables is not None:  # prefix cache: keys come from the pages
                return K.prefill_attention(q, k_cache, v_cache, ctx.cu_seqlens_q, ctx.cu_seqlens_k,
                                           ctx.max_seqlen_q, self.scale, block_tables=ctx.block_tables)
            return K.prefill_attention(q, k, v, ctx.cu_seqlens_q, ctx.cu_seqlens_k, ctx.max_seqlen_q, self.scale)
        return K.paged_decode_attention(q, k_cache, v_cache, ctx.block_tables, ctx.context_lens, self.scale)
