"""ERNIE 4.5 dense model on the kavor_b200 layers (drop-in for kavor/models/ernie4_5.py).

The attention (ernie4_5.py:43-114) differs from Qwen3's in three ways: no q/k
RMSNorm, a q/k/v projection bias when the config's ``use_bias`` is set, and
the interleaved RoPE (pairs (2i, 2i+1), ernie4_5.py:82-88; rotary_embedding.py:68-79),
which the fused prologue kernel applies in place of the neox rotation. The LM
head shares the embedding when ``tie_word_embeddings`` is set (:195-196).

Residual wiring: the reference layer (ernie4_5.py:130-148) adds the residual
in bf16 and then normalises that sum (``norm(residual + h)``); this package
runs the same steps as one fused add+RMSNorm, which keeps the bf16 sum as the
new residual (bit-identical to the reference's) and normalises the fp32 sum
before its bf16 rounding. The normalised activations therefore agree with
the reference's to within one bf16 rounding of the norm's input.
"""
from __future__ import annotations

from kavor_b200.models.qwen3 import Qwen3Attention, Qwen3DecoderLayer, Qwen3ForCausalLM, Qwen3Model, rope_theta_of


class Ernie4_5DecoderLayer(Qwen3DecoderLayer):

    @staticmethod
    def make_attention(config) -> Qwen3Attention:
        """ernie4_5.py:46-95."""
        return Qwen3Attention(
            hidden_size=config.hidden_size,
            num_heads=config.num_attention_heads,
            num_kv_heads=config.num_key_value_heads,
            max_position=config.max_position_embeddings,
            rms_norm_eps=config.rms_norm_eps,
            qkv_bias=bool(config.use_bias),
            head_dim=getattr(config, "head_dim", None),
            rope_theta=rope_theta_of(config, default=1000000.0),
            qk_norm=False,
            rope_interleaved=True,
        )

    @staticmethod
    def attention_layout(config) -> dict:
        return dict(qk_norm=False, qkv_bias=bool(config.use_bias))


class Ernie4_5Model(Qwen3Model):
    layer_cls = Ernie4_5DecoderLayer


class Ernie4_5ForCausalLM(Qwen3ForCausalLM):
    model_cls = Ernie4_5Model
