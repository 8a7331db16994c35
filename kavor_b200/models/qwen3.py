"""Qwen3 dense model on the kavor_b200 layers (drop-in for kavor/models/qwen3.py).

Module tree, parameter names and the packed checkpoint mapping are those of
qwen3.py:14-219, so reference checkpoints load unchanged. The forward is the
same computation with the per-layer work fused into fewer kernels:

* attention prologue (qwen3.py:80-89 + flash_attention_kvcache.py:72): after
  the QKV GEMM, ONE kernel does q_norm, k_norm, RoPE on q and k and writes the
  k/v rows into the paged cache, in place on the packed qkv rows;
* attention: paged decode / varlen prefill kernels;
* residual wiring (qwen3.py:149-162) with fused add+RMSNorm after every
  row-parallel projection.
"""
from __future__ import annotations

import contextlib

import torch
from torch import nn

from kavor_b200 import _kernels as K
from kavor_b200.layers.activation import SiluAndMul
from kavor_b200.layers.allreduce import get_decode_microbatches, get_tp_allreduce
from kavor_b200.layers.attention import Attention
from kavor_b200.layers.embed_head import ParallelLMHead, VocabParallelEmbedding
from kavor_b200.layers.layernorm import RMSNorm
from kavor_b200.layers.linear import (MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear, _tp,
                                      gate_up_silu)
from kavor_b200.layers.rotary_embedding import get_rope
from kavor_b200.utils.context import context_scope, decode_rows, get_context


def rope_theta_of(config, default: float = 1000000.0) -> float:
    """rope theta from either the flat field or the rope_scaling/rope_parameters dict
    (qwen3.py:57-58, :138-139)."""
    theta = getattr(config, "rope_theta", None)
    for name in ("rope_scaling", "rope_parameters"):
        d = getattr(config, name, None)
        if isinstance(d, dict) and "rope_theta" in d:
            theta = d["rope_theta"]
    return float(theta if theta is not None else default)


class Qwen3Attention(nn.Module):

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, max_position: int = 4096 * 32,
                 head_dim: int | None = None, rms_norm_eps: float = 1e-06, qkv_bias: bool = False,
                 rope_theta: float = 10000, rope_scaling: dict | None = None, qk_norm: bool | None = None,
                 rope_interleaved: bool = False) -> None:
        super().__init__()
        _, tp_size = _tp()
        if num_heads % tp_size or num_kv_heads % tp_size:
            raise ValueError("attention heads must be divisible by the tensor-parallel size")
        self.total_num_heads = num_heads
        self.num_heads = num_heads // tp_size
        self.total_num_kv_heads = num_kv_heads
        self.num_kv_heads = num_kv_heads // tp_size
        self.head_dim = head_dim or hidden_size // num_heads
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.scaling = self.head_dim ** -0.5
        self.qkv_bias = qkv_bias
        # Qwen3 normalises q and k exactly when the projection has no bias
        # (qwen3.py:71-73, :136); the other dense families choose explicitly
        self.qk_norm = (not qkv_bias) if qk_norm is None else qk_norm
        self.rms_norm_eps = rms_norm_eps
        self.qkv_proj = QKVParallelLinear((num_heads + 2 * num_kv_heads) * self.head_dim, hidden_size,
                                          self.head_dim, num_heads, num_kv_heads, bias=qkv_bias)
        self.o_proj = RowParallelLinear(num_heads * self.head_dim, hidden_size, bias=False)
        if isinstance(rope_scaling, dict):
            rope_theta = rope_scaling.get("rope_theta", rope_theta)
        self.rotary_emb = get_rope(self.head_dim, rotary_dim=self.head_dim, max_position=max_position,
                                   base=rope_theta, interleaved=rope_interleaved)
        self.attn = Attention(self.num_heads, self.head_dim, self.scaling, self.num_kv_heads)
        if self.qk_norm:
            self.q_norm = RMSNorm(self.head_dim, eps=rms_norm_eps)
            self.k_norm = RMSNorm(self.head_dim, eps=rms_norm_eps)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor, reduce: bool = True,
                out: torch.Tensor | None = None, attention_turn=None) -> torch.Tensor:
        """``attention_turn``: an optional context manager entered around the
        attention kernel alone (a decode step split into micro-batches orders
        the halves' attention kernels with it)."""
        qkv = self.qkv_proj(hidden_states)
        ctx = get_context()
        k_cache, v_cache = self.attn.k_cache[0], self.attn.v_cache[0]
        has_cache = k_cache.numel() > 0
        K.qknorm_rope_store(
            qkv, self.num_heads, self.num_kv_heads, self.head_dim,
            self.q_norm.weight if self.qk_norm else None, self.k_norm.weight if self.qk_norm else None,
            self.rms_norm_eps, positions, self.rotary_emb.cos_sin_cache, self.rotary_emb.interleaved,
            k_cache if has_cache else None, v_cache if has_cache else None,
            ctx.slot_mapping if has_cache else None)
        q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
        q = q.view(-1, self.num_heads, self.head_dim)
        k = k.view(-1, self.num_kv_heads, self.head_dim)
        v = v.view(-1, self.num_kv_heads, self.head_dim)
        with attention_turn if attention_turn is not None else contextlib.nullcontext():
            o = self.attn(q, k, v, kv_stored=True)
        return self.o_proj(o.flatten(1, -1), reduce=reduce, out=out)


class Qwen3MLP(nn.Module):

    def __init__(self, hidden_size: int, intermediate_size: int, hidden_act: str) -> None:
        super().__init__()
        if hidden_act != "silu":
            raise ValueError(f"unsupported activation {hidden_act!r}")
        self.gate_up_proj = MergedColumnParallelLinear(hidden_size, [intermediate_size] * 2, bias=False)
        self.down_proj = RowParallelLinear(intermediate_size, hidden_size, bias=False)
        self.act_fn = SiluAndMul()

    def forward(self, x: torch.Tensor, reduce: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
        h = gate_up_silu(x, self.gate_up_proj.weight)  # gate-up projection and SiluAndMul in one kernel
        if h is None:
            h = self.act_fn(self.gate_up_proj(x))
        return self.down_proj(h, reduce=reduce, out=out)


class Qwen3DecoderLayer(nn.Module):

    def __init__(self, config) -> None:
        super().__init__()
        self.self_attn = self.make_attention(config)
        self.mlp = Qwen3MLP(config.hidden_size, config.intermediate_size, config.hidden_act)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    @staticmethod
    def make_attention(config) -> Qwen3Attention:
        """qwen3.py:130-140."""
        return Qwen3Attention(
            hidden_size=config.hidden_size,
            num_heads=config.num_attention_heads,
            num_kv_heads=config.num_key_value_heads,
            max_position=config.max_position_embeddings,
            rms_norm_eps=config.rms_norm_eps,
            qkv_bias=getattr(config, "attention_bias", True),
            head_dim=getattr(config, "head_dim", None),
            rope_theta=rope_theta_of(config),
            rope_scaling=None,
        )

    @staticmethod
    def attention_layout(config) -> dict:
        """Which optional attention tensors the checkpoint holds."""
        bias = getattr(config, "attention_bias", True)
        return dict(qk_norm=not bias, qkv_bias=bias)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor,
                residual: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
        if residual is None:
            hidden_states, residual = self.input_layernorm(hidden_states), hidden_states
        else:
            hidden_states, residual = self.input_layernorm(hidden_states, residual)
        hidden_states = self.self_attn(positions, hidden_states)
        hidden_states, residual = self.post_attention_layernorm(hidden_states, residual)
        hidden_states = self.mlp(hidden_states)
        return hidden_states, residual


class Qwen3Model(nn.Module):
    layer_cls = Qwen3DecoderLayer

    def __init__(self, config) -> None:
        super().__init__()
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([self.layer_cls(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        ar = get_tp_allreduce()
        if ar is not None and self.embed_tokens.tp_size > 1:
            mb = get_decode_microbatches()
            if mb is not None and not get_context().is_prefill and mb.applies(input_ids.numel()):
                return self._forward_microbatched(mb, input_ids, positions)
            return self._forward_fused_allreduce(ar, input_ids, positions)
        hidden_states = self.embed_tokens(input_ids)
        residual = None
        for layer in self.layers:
            hidden_states, residual = layer(positions, hidden_states, residual)
        hidden_states, _ = self.norm(hidden_states, residual)
        return hidden_states

    def _forward_fused_allreduce(self, ar, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """TP > 1: every all-reduce is fused with the add+RMSNorm after it; the
        embedding and the row-parallel projections write their rank-local
        partial sums straight into the communicator's NVLink-visible buffers."""
        T = input_ids.numel()
        ar.start_forward()
        idx = ar.EMBED_BUFFER
        self.embed_tokens(input_ids, reduce=False, out=ar.partial_buffer(idx, T))
        residual = None
        for layer in self.layers:
            ln = layer.input_layernorm
            x, residual = ar.reduce_norm(idx, T, residual, ln.weight, ln.eps)
            idx, buf = ar.next_buffer(T)
            layer.self_attn(positions, x, reduce=False, out=buf)
            ln = layer.post_attention_layernorm
            x, residual = ar.reduce_norm(idx, T, residual, ln.weight, ln.eps)
            idx, buf = ar.next_buffer(T)
            layer.mlp(x, reduce=False, out=buf)
        out, _ = ar.reduce_norm(idx, T, residual, self.norm.weight, self.norm.eps)
        return out

    def _forward_microbatched(self, mb, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """A TP > 1 decode step as two micro-batches (``DecodeMicrobatches``):
        the same per-row computation as ``_forward_fused_allreduce``, issued
        layer by layer for rows [0, h) on the launching stream and rows [h, T)
        on the second stream, each half with its own communicator and its
        slices of the step's metadata; the halves' attention kernels take
        turns. Returns the final normalised rows of both halves in one
        [T, hidden] tensor."""
        T = input_ids.numel()
        spans = mb.spans(T)
        ctx = get_context()
        subs = [decode_rows(ctx, lo, hi) for lo, hi in spans]
        out = torch.empty(T, self.embed_tokens.weight.shape[1], dtype=torch.bfloat16, device=input_ids.device)
        mb.fork()
        state = []  # per half: [partial buffer index, residual]
        for m, (lo, hi) in enumerate(spans):
            ar = mb.comms[m]
            with mb.on(m):
                ar.start_forward()
                self.embed_tokens(input_ids[lo:hi], reduce=False, out=ar.partial_buffer(ar.EMBED_BUFFER, hi - lo))
            state.append([ar.EMBED_BUFFER, None])
        for layer in self.layers:
            for m, (lo, hi) in enumerate(spans):
                ar, st, n = mb.comms[m], state[m], hi - lo
                with mb.on(m), context_scope(subs[m]):
                    ln = layer.input_layernorm
                    x, st[1] = ar.reduce_norm(st[0], n, st[1], ln.weight, ln.eps)
                    st[0], buf = ar.next_buffer(n)
                    layer.self_attn(positions[lo:hi], x, reduce=False, out=buf, attention_turn=mb.attention_turn(m))
            for m, (lo, hi) in enumerate(spans):
                ar, st, n = mb.comms[m], state[m], hi - lo
                with mb.on(m):
                    ln = layer.post_attention_layernorm
                    x, st[1] = ar.reduce_norm(st[0], n, st[1], ln.weight, ln.eps)
                    st[0], buf = ar.next_buffer(n)
                    layer.mlp(x, reduce=False, out=buf)
        for m, (lo, hi) in enumerate(spans):
            ar, st = mb.comms[m], state[m]
            with mb.on(m):
                y, _ = ar.reduce_norm(st[0], hi - lo, st[1], self.norm.weight, self.norm.eps)
                out[lo:hi].copy_(y)
        mb.join()
        return out


class Qwen3ForCausalLM(nn.Module):
    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", 0),
        "up_proj": ("gate_up_proj", 1),
    }

    model_cls = Qwen3Model

    def __init__(self, config) -> None:
        super().__init__()
        self.model = self.model_cls(config)
        self.lm_head = ParallelLMHead(config.vocab_size, config.hidden_size)
        if self.ties_word_embeddings(config):
            self.lm_head.weight.data = self.model.embed_tokens.weight.data

    @staticmethod
    def ties_word_embeddings(config) -> bool:
        """qwen3.py:205-206: the LM head shares the embedding when the config says so."""
        return bool(getattr(config, "tie_word_embeddings", False))

    @classmethod
    def attention_layout(cls, config) -> dict:
        return cls.model_cls.layer_cls.attention_layout(config)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids, positions)

    def compute_logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return self.lm_head(hidden_states)
