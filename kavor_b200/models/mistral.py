"""Mistral dense model on the kavor_b200 layers (drop-in for kavor/models/mistral.py).

The same decoder as Qwen3 (residual wiring mistral.py:108-121, MLP :13-35,
model :123-145) with three differences in the attention (mistral.py:37-97):
no q/k RMSNorm, no projection bias, and the rope theta of the config (10000
when it names none). The LM head never shares the embedding (mistral.py:162).
Module and parameter names are the reference's, so its checkpoints load
unchanged; the fused prologue kernel runs with the norm step off.
"""
from __future__ import annotations

from kavor_b200.models.qwen3 import Qwen3Attention, Qwen3DecoderLayer, Qwen3ForCausalLM, Qwen3Model, rope_theta_of


class MistralDecoderLayer(Qwen3DecoderLayer):

    @staticmethod
    def make_attention(config) -> Qwen3Attention:
        """mistral.py:39-82."""
        return Qwen3Attention(
            hidden_size=config.hidden_size,
            num_heads=config.num_attention_heads,
            num_kv_heads=config.num_key_value_heads,
            max_position=config.max_position_embeddings,
            rms_norm_eps=config.rms_norm_eps,
            qkv_bias=False,
            head_dim=getattr(config, "head_dim", None),
            rope_theta=rope_theta_of(config, default=10000.0),
            qk_norm=False,
        )

    @staticmethod
    def attention_layout(config) -> dict:
        return dict(qk_norm=False, qkv_bias=False)


class MistralModel(Qwen3Model):
    layer_cls = MistralDecoderLayer


class MistralForCausalLM(Qwen3ForCausalLM):
    model_cls = MistralModel

    @staticmethod
    def ties_word_embeddings(config) -> bool:
        return False
