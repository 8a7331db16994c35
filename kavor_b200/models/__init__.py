"""Model registry and weight loading (drop-in for kavor/models/modeling_auto.py).

``AutoModelForCausalLM.from_pretrained(hf_config, use_tqdm, load_format)``
builds the registered model class for ``hf_config.model_type`` and fills its
parameters through the per-parameter ``weight_loader`` of the TP layers:

* ``load_format="auto"``: the safetensors (or ``.bin``) files of the model
  directory, checkpoint names mapped through ``packed_modules_mapping``
  (modeling_auto.py:49-131), then a missing-parameter check (:150-162);
* ``load_format="dummy"``: a synthetic checkpoint with the reference
  checkpoint's tensor names and FULL (unsharded) shapes, every tensor drawn on
  the target device from its own seeded generator: matrices N(0, 0.02), norm
  gains N(1, 0.1), projection biases N(0, 0.5) (the size of the projections'
  outputs, so a bias visibly moves them). Because it goes through the same TP
  loaders, a TP=N model is exactly the TP=1 model sharded.
"""
from __future__ import annotations

import glob
import os
import zlib

import torch
from torch import nn

from kavor_b200.models.ernie4_5 import Ernie4_5ForCausalLM
from kavor_b200.models.mistral import MistralForCausalLM
from kavor_b200.models.qwen3 import Qwen3ForCausalLM

# model_type -> class (model_mapping.py:6-15, the dense text families)
MODEL_REGISTRY: dict[str, type[nn.Module]] = {
    "qwen3": Qwen3ForCausalLM,
    "mistral": MistralForCausalLM,
    "ernie4_5": Ernie4_5ForCausalLM,
}


def _assign(model: nn.Module, name: str, tensor: torch.Tensor, packed: dict, loaded: set[str]) -> None:
    for key, (target, shard_id) in packed.items():
        if key in name:
            pname = name.replace(key, target)
            param = model.get_parameter(pname)
            param.weight_loader(param, tensor, shard_id)
            loaded.add(pname)
            return
    param = model.get_parameter(name)
    loader = getattr(param, "weight_loader", None)
    if loader is None:
        param.data.copy_(tensor)
    else:
        loader(param, tensor)
    loaded.add(name)


def synthetic_checkpoint(config, seed: int, device: torch.device):
    """Yield (name, full tensor) of a checkpoint of the config's model family
    (q/k norm gains or q/k/v biases as that family's attention has them) with
    random values."""
    layout = AutoModelForCausalLM.model_class(config).attention_layout(config)
    tie = AutoModelForCausalLM.model_class(config).ties_word_embeddings(config)
    H, I = config.hidden_size, config.intermediate_size
    hd = getattr(config, "head_dim", None) or H // config.num_attention_heads
    Hq, Hkv = config.num_attention_heads, config.num_key_value_heads
    dtype = torch.bfloat16

    def draw(name: str, shape, mean: float, std: float) -> torch.Tensor:
        g = torch.Generator(device=device)
        g.manual_seed((zlib.crc32(name.encode()) ^ (seed * 0x9E3779B1)) & 0xFFFFFFFFFFFF)
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        return t.mul_(std).add_(mean).to(dtype)

    yield "model.embed_tokens.weight", draw("model.embed_tokens.weight", (config.vocab_size, H), 0.0, 0.02)
    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        for n, shape in (("self_attn.q_proj.weight", (Hq * hd, H)), ("self_attn.k_proj.weight", (Hkv * hd, H)),
                         ("self_attn.v_proj.weight", (Hkv * hd, H)), ("self_attn.o_proj.weight", (H, Hq * hd)),
                         ("mlp.gate_proj.weight", (I, H)), ("mlp.up_proj.weight", (I, H)),
                         ("mlp.down_proj.weight", (H, I))):
            yield p + n, draw(p + n, shape, 0.0, 0.02)
        if layout["qk_norm"]:
            for n in ("self_attn.q_norm.weight", "self_attn.k_norm.weight"):
                yield p + n, draw(p + n, (hd,), 1.0, 0.1)
        if layout["qkv_bias"]:
            for n, size in (("self_attn.q_proj.bias", Hq * hd), ("self_attn.k_proj.bias", Hkv * hd),
                            ("self_attn.v_proj.bias", Hkv * hd)):
                yield p + n, draw(p + n, (size,), 0.0, 0.5)
        for n in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            yield p + n, draw(p + n, (H,), 1.0, 0.1)
    yield "model.norm.weight", draw("model.norm.weight", (H,), 1.0, 0.1)
    if not tie:
        yield "lm_head.weight", draw("lm_head.weight", (config.vocab_size, H), 0.0, 0.02)


def _checkpoint_files(path: str):
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if files:
        from safetensors import safe_open

        for f in files:
            with safe_open(f, framework="pt", device="cpu") as fh:
                for name in fh.keys():
                    yield name, fh.get_tensor(name)
        return
    files = sorted(glob.glob(os.path.join(path, "*.bin")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors or *.bin weights in {path} (use load_format='dummy')")
    for f in files:
        for name, t in torch.load(f, map_location="cpu", weights_only=True).items():
            yield name, t


class AutoModelForCausalLM:

    @classmethod
    def model_class(cls, hf_config) -> type[nn.Module]:
        model_type = getattr(hf_config, "model_type", None)
        if model_type not in MODEL_REGISTRY:
            raise ValueError(f"model_type {model_type!r} is not supported (registered: {sorted(MODEL_REGISTRY)})")
        return MODEL_REGISTRY[model_type]

    @classmethod
    def from_pretrained(cls, hf_config, use_tqdm: bool = False, load_format: str = "auto", seed: int = 0,
                        **kwargs) -> nn.Module:
        model = cls.model_class(hf_config)(hf_config)
        cls.load_weight(model, hf_config, load_format=load_format, seed=seed)
        return model

    @classmethod
    @torch.inference_mode()
    def load_weight(cls, model: nn.Module, hf_config, load_format: str = "auto", seed: int = 0) -> None:
        packed = getattr(model, "packed_modules_mapping", {})
        device = next(model.parameters()).device
        if load_format == "dummy":
            source = synthetic_checkpoint(hf_config, seed, device)
        elif load_format == "auto":
            source = _checkpoint_files(hf_config.name_or_path)
        else:
            raise ValueError(f"unknown load_format {load_format!r}")
        loaded: set[str] = set()
        for name, tensor in source:
            _assign(model, name, tensor, packed, loaded)
        params = {n for n, _ in model.named_parameters()}
        if model.ties_word_embeddings(hf_config):
            loaded.add("lm_head.weight")
        missing = sorted(params - loaded)
        if missing:
            raise RuntimeError(f"{len(missing)} parameters were not loaded, e.g. {missing[:5]}")
