"""Weight loading from checkpoint files (modeling_auto.py:49-162 of the
reference) on the CPU: a checkpoint written with the reference's tensor names
(separate q/k/v and gate/up projections) loads through the packed-module
mapping and the TP weight loaders into exactly the parameters that the
seeded dummy checkpoint gives; safetensors shards and a .bin file both load;
a checkpoint missing a tensor and an unknown model type are refused."""
import pytest
import torch

from kavor_b200.config import load_hf_config, write_model_dir


def _build(hf):
    from kavor_b200.models import AutoModelForCausalLM

    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        return AutoModelForCausalLM.model_class(hf)(hf)
    finally:
        torch.set_default_dtype(prev)


def _tiny(tmp_path, preset="Qwen3-0.6B", **kw):
    shape = dict(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=1024)
    shape.update(kw)
    return load_hf_config(write_model_dir(str(tmp_path / "m"), preset, **shape))


def _checkpoint(hf):
    from kavor_b200.models import synthetic_checkpoint

    return dict(synthetic_checkpoint(hf, seed=11, device=torch.device("cpu")))


def _params(model):
    return {n: p.detach().clone() for n, p in model.named_parameters()}


@pytest.mark.parametrize("preset", ["Qwen3-0.6B", "Qwen3-8B", "Mistral-7B-v0.3", "ERNIE-4.5-0.3B"])
def test_safetensors_shards_load_like_the_dummy_checkpoint(tmp_path, preset):
    from safetensors.torch import save_file

    from kavor_b200.models import AutoModelForCausalLM

    hf = _tiny(tmp_path, preset)
    ckpt = _checkpoint(hf)
    names = sorted(ckpt)
    half = len(names) // 2
    save_file({n: ckpt[n].contiguous() for n in names[:half]}, str(tmp_path / "m" / "model-00001.safetensors"))
    save_file({n: ckpt[n].contiguous() for n in names[half:]}, str(tmp_path / "m" / "model-00002.safetensors"))
    from_files = _build(hf)
    AutoModelForCausalLM.load_weight(from_files, hf, load_format="auto")
    dummy = _build(hf)
    AutoModelForCausalLM.load_weight(dummy, hf, load_format="dummy", seed=11)
    a, b = _params(from_files), _params(dummy)
    assert a.keys() == b.keys()
    for n in a:
        assert torch.equal(a[n], b[n]), n
    # the merged projections hold the checkpoint's rows in [q | k | v] and [gate | up] order
    qkv = a["model.layers.1.self_attn.qkv_proj.weight"]
    q, k, v = (ckpt[f"model.layers.1.self_attn.{n}_proj.weight"] for n in "qkv")
    assert torch.equal(qkv, torch.cat([q, k, v]))
    gu = a["model.layers.0.mlp.gate_up_proj.weight"]
    assert torch.equal(gu, torch.cat([ckpt["model.layers.0.mlp.gate_proj.weight"],
                                      ckpt["model.layers.0.mlp.up_proj.weight"]]))


def test_a_bin_checkpoint_loads(tmp_path):
    from kavor_b200.models import AutoModelForCausalLM

    hf = _tiny(tmp_path)
    ckpt = _checkpoint(hf)
    torch.save(ckpt, str(tmp_path / "m" / "pytorch_model.bin"))
    model = _build(hf)
    AutoModelForCausalLM.load_weight(model, hf, load_format="auto")
    assert torch.equal(model.get_parameter("model.norm.weight"), ckpt["model.norm.weight"])


def test_a_missing_tensor_is_reported(tmp_path):
    from safetensors.torch import save_file

    from kavor_b200.models import AutoModelForCausalLM

    hf = _tiny(tmp_path)
    ckpt = _checkpoint(hf)
    del ckpt["model.layers.1.post_attention_layernorm.weight"]
    save_file(ckpt, str(tmp_path / "m" / "model.safetensors"))
    with pytest.raises(RuntimeError, match="not loaded"):
        AutoModelForCausalLM.load_weight(_build(hf), hf, load_format="auto")


def test_no_weights_and_unknown_families_are_refused(tmp_path):
    from kavor_b200.models import AutoModelForCausalLM

    hf = _tiny(tmp_path)
    with pytest.raises(FileNotFoundError, match="load_format='dummy'"):
        AutoModelForCausalLM.load_weight(_build(hf), hf, load_format="auto")
    hf.model_type = "qwen3_5"
    with pytest.raises(ValueError, match="not supported"):
        AutoModelForCausalLM.model_class(hf)
