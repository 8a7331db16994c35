"""Dense decoder forward (Qwen3, Mistral, ERNIE 4.5) on the CPU oracle ops
(test infrastructure).

Composes oracle.ops with the reference wiring:
decoder layer qwen3.py:149-162, attention qwen3.py:75-91, MLP :116-120,
model :176-186, LM head embed_head.py:56-66. The other dense families differ
only in the flags of ``Shape``: Mistral (mistral.py:84-97) has neither q/k
norm nor bias; ERNIE 4.5 (ernie4_5.py:97-148) has no q/k norm, an optional
q/k/v bias, the interleaved RoPE, and adds its residual in bf16 before a plain
RMSNorm (``separate_residual_add``) where the other two use the fused
add+RMSNorm. Weights come as a dict keyed by the reference checkpoint names
(q_proj/k_proj/... unpacked, full TP=1 shapes).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from oracle import ops


@dataclass
class Shape:
    hidden: int
    inter: int
    layers: int
    hq: int
    hkv: int
    head_dim: int = 128
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1e6
    tie: bool = False
    qk_norm: bool = True
    qkv_bias: bool = False
    interleaved: bool = False
    separate_residual_add: bool = False


@dataclass
class Batch:
    """One step's metadata (the reference Context, model_runner.py:385-473)."""
    is_prefill: bool
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None


def attention(p: dict, pre: str, x: torch.Tensor, batch: Batch, caches, shape: Shape, cache) -> torch.Tensor:
    hd = shape.head_dim
    bias = None
    if shape.qkv_bias:
        bias = torch.cat([p[pre + "q_proj.bias"], p[pre + "k_proj.bias"], p[pre + "v_proj.bias"]])
    qkv = ops.linear(x, torch.cat([p[pre + "q_proj.weight"], p[pre + "k_proj.weight"], p[pre + "v_proj.weight"]]),
                     bias)
    q, k, v = qkv.split([shape.hq * hd, shape.hkv * hd, shape.hkv * hd], dim=-1)
    q = q.reshape(-1, shape.hq, hd)
    k = k.reshape(-1, shape.hkv, hd)
    v = v.reshape(-1, shape.hkv, hd)
    if shape.qk_norm:
        q = ops.rmsnorm(q, p[pre + "q_norm.weight"], shape.eps)
        k = ops.rmsnorm(k, p[pre + "k_norm.weight"], shape.eps)
    q = ops.rope(q, batch.positions, cache, shape.interleaved)
    k = ops.rope(k, batch.positions, cache, shape.interleaved)
    k_cache, v_cache = caches
    ops.store_kvcache(k, v, k_cache, v_cache, batch.slot_mapping)
    scale = hd ** -0.5
    if batch.is_prefill:
        if batch.block_tables is not None:
            o = ops.varlen_prefill_attention(q, k_cache, v_cache, batch.cu_seqlens_q, batch.cu_seqlens_k, scale,
                                             batch.block_tables)
        else:
            o = ops.varlen_prefill_attention(q, k, v, batch.cu_seqlens_q, batch.cu_seqlens_k, scale)
    else:
        o = ops.paged_decode_attention(q, k_cache, v_cache, batch.block_tables, batch.context_lens, scale)
    return ops.linear(o.reshape(o.shape[0], -1), p[pre + "o_proj.weight"])


def _add_norm(h: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, shape: Shape):
    """(normed, new residual). Fused add+RMSNorm (qwen3.py:158-160), or, for
    ERNIE 4.5, the bf16 sum and then an RMSNorm of it (ernie4_5.py:136-147)."""
    if shape.separate_residual_add:
        s = residual + h
        return ops.rmsnorm(s, weight, shape.eps), s
    return ops.add_rmsnorm(h, residual, weight, shape.eps)


def decoder_layer(p: dict, i: int, h: torch.Tensor, residual, batch: Batch, caches, shape: Shape, cache):
    pre = f"model.layers.{i}."
    if residual is None:
        x, residual = ops.rmsnorm(h, p[pre + "input_layernorm.weight"], shape.eps), h
    else:
        x, residual = _add_norm(h, residual, p[pre + "input_layernorm.weight"], shape)
    h = attention(p, pre + "self_attn.", x, batch, caches, shape, cache)
    x, residual = _add_norm(h, residual, p[pre + "post_attention_layernorm.weight"], shape)
    gu = ops.linear(x, torch.cat([p[pre + "mlp.gate_proj.weight"], p[pre + "mlp.up_proj.weight"]]))
    h = ops.linear(ops.silu_mul(gu), p[pre + "mlp.down_proj.weight"])
    return h, residual


def forward(p: dict, input_ids: torch.Tensor, batch: Batch, kv: list, shape: Shape, max_position: int = 40960):
    """Returns (final hidden states [T, H], logits [B, vocab] of the last token per sequence)."""
    cache = ops.cos_sin_cache(shape.head_dim, max_position, shape.rope_theta)
    h = ops.embedding(input_ids, p["model.embed_tokens.weight"])
    residual = None
    for i in range(shape.layers):
        h, residual = decoder_layer(p, i, h, residual, batch, kv[i], shape, cache)
    h, _ = _add_norm(h, residual, p["model.norm.weight"], shape)
    last = h
    if batch.is_prefill:
        last = h[batch.cu_seqlens_q[1:].long() - 1]
    head = p["model.embed_tokens.weight"] if shape.tie else p["lm_head.weight"]
    return h, ops.linear(last, head)
