"""The reference's decoder-layer arithmetic evaluated on the GPU (test
infrastructure, used by the GPU parity tests as a second checker beside the
CPU fixtures).

Where the reference calls a library, this calls the same library on the same
GPU: ``F.linear`` (cuBLAS) for every projection (linear.py:50,73,157) and
``flash_attn_with_kvcache`` for decode attention
(flash_attention_kvcache.py:81-83, flash-attn 2.8.3 run, never read). The
reference's own Triton / compiled kernels (RMSNorm layernorm.py:8-39,
add+RMSNorm :114-140, RoPE rotary_embedding.py:8-53, SiluAndMul
activation.py:8-11) are their fp32 restatements from ``oracle.ops`` applied
to CUDA tensors, and store_kvcache (flash_attention_kvcache.py:23-34) is an
indexed copy. So the only arithmetic differences left against the product's
kernels are accumulation orders, not the CPU's fp32 GEMM against the GPU's.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import ops


def flash_attn_or_none():
    """The flash-attn module when it imports and has a kernel for this GPU."""
    try:
        import flash_attn
    except ImportError:
        return None
    q = torch.randn(1, 1, 8, 128, device="cuda", dtype=torch.bfloat16)
    kc = torch.randn(1, 256, 8, 128, device="cuda", dtype=torch.bfloat16)
    try:
        flash_attn.flash_attn_with_kvcache(q, kc, kc, cache_seqlens=torch.ones(1, dtype=torch.int32, device="cuda"),
                                           block_table=torch.zeros(1, 1, dtype=torch.int32, device="cuda"),
                                           causal=True)
        torch.cuda.synchronize()
    except RuntimeError:
        return None
    return flash_attn


def decode_layer(fa, weights: dict, shape: dict, hidden, residual, positions, slot_mapping, context_lens,
                 block_tables, k_cache, v_cache, max_position: int = 40960):
    """One Qwen3 decoder layer, one decode step (qwen3.py:149-162), every
    tensor on the GPU. ``weights`` are the layer's checkpoint tensors (q_proj,
    k_proj, ... unpacked); the caches are updated in place. Returns
    (hidden, residual) as the reference layer returns them."""
    hd, hq, hkv = shape["head_dim"], shape["num_attention_heads"], shape["num_key_value_heads"]
    eps = shape.get("rms_norm_eps", 1e-6)
    w = {k: v.cuda() for k, v in weights.items()}
    if residual is None:
        x, residual = ops.rmsnorm(hidden, w["input_layernorm.weight"], eps), hidden
    else:
        x, residual = ops.add_rmsnorm(hidden, residual, w["input_layernorm.weight"], eps)
    qkv = F.linear(x, torch.cat([w["self_attn.q_proj.weight"], w["self_attn.k_proj.weight"],
                                 w["self_attn.v_proj.weight"]]))
    q, k, v = qkv.split([hq * hd, hkv * hd, hkv * hd], dim=-1)
    q = ops.rmsnorm(q.reshape(-1, hq, hd), w["self_attn.q_norm.weight"], eps)
    k = ops.rmsnorm(k.reshape(-1, hkv, hd), w["self_attn.k_norm.weight"], eps)
    cache = ops.cos_sin_cache(hd, max_position, shape.get("rope_theta", 1e6)).cuda()
    q, k = ops.rope(q, positions, cache), ops.rope(k, positions, cache)
    v = v.reshape(-1, hkv, hd)
    bs = k_cache.shape[1]
    ok = slot_mapping >= 0
    sl = slot_mapping[ok].long()
    k_cache[sl // bs, sl % bs] = k[ok]
    v_cache[sl // bs, sl % bs] = v[ok]
    tables = block_tables.clamp(min=0)  # flash-attn reads the padding entries too
    o = fa.flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache, cache_seqlens=context_lens,
                                   block_table=tables, softmax_scale=hd ** -0.5, causal=True).squeeze(1)
    h = F.linear(o.reshape(o.shape[0], -1), w["self_attn.o_proj.weight"])
    x, residual = ops.add_rmsnorm(h, residual, w["post_attention_layernorm.weight"], eps)
    gu = F.linear(x, torch.cat([w["mlp.gate_proj.weight"], w["mlp.up_proj.weight"]]))
    h = F.linear(ops.silu_mul(gu), w["mlp.down_proj.weight"])
    return h, residual
