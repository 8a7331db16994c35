"""Config (config.py:16-53 of the reference) on the CPU: the reference's checks
(model directory, block size a multiple of 256, TP size 1..8), max_model_len
capped by the checkpoint's max_position_embeddings, and this package's own
options validated before anything is built."""
import pytest

from kavor_b200.config import FAMILY_PRESETS, QWEN3_PRESETS, Config, load_hf_config, write_model_dir


@pytest.fixture
def model_dir(tmp_path):
    return write_model_dir(str(tmp_path / "m"), "Qwen3-0.6B", max_position_embeddings=2048)


def test_defaults_and_length_cap(model_dir):
    cfg = Config(model_dir, load_format="dummy", max_model_len=4096, rdzv_port=12345)
    assert cfg.max_model_len == 2048  # the checkpoint's max_position_embeddings
    assert cfg.kvcache_block_size == 256 and cfg.gemm_backend == "auto" and cfg.rdzv_port == 12345
    assert cfg.hf_config.hidden_size == QWEN3_PRESETS["Qwen3-0.6B"]["hidden_size"]
    assert Config(model_dir, max_model_len=1000).max_model_len == 1000


def test_a_free_port_is_picked_when_none_is_given(model_dir, monkeypatch):
    monkeypatch.delenv("KAVOR_RDZV_PORT", raising=False)
    assert 0 < Config(model_dir).rdzv_port < 65536
    monkeypatch.setenv("KAVOR_RDZV_PORT", "23456")
    assert Config(model_dir).rdzv_port == 23456


@pytest.mark.parametrize("kwargs", [
    {"kvcache_block_size": 128},
    {"tensor_parallel_size": 0},
    {"tensor_parallel_size": 9},
    {"load_format": "safetensors"},
    {"gemm_backend": "triton"},
    {"gemm_l2_prefetch": 65},
    {"decode_microbatches": 3},
    {"decode_microbatch_min_bs": 1},
])
def test_invalid_options_are_rejected(model_dir, kwargs):
    with pytest.raises(AssertionError):
        Config(model_dir, **kwargs)


def test_missing_model_directory(tmp_path):
    with pytest.raises(RuntimeError, match="Model not found"):
        Config(str(tmp_path / "absent"))


@pytest.mark.parametrize("preset", sorted(QWEN3_PRESETS) + sorted(FAMILY_PRESETS))
def test_written_model_directories_parse(tmp_path, preset):
    """Every preset's config.json reads back through transformers with the
    preset's shapes (the dummy-weight runs and the benches depend on it)."""
    d = write_model_dir(str(tmp_path / preset), preset, num_hidden_layers=2)
    hf = load_hf_config(d)
    shapes = QWEN3_PRESETS.get(preset) or FAMILY_PRESETS[preset]
    for key in ("hidden_size", "intermediate_size", "num_attention_heads", "num_key_value_heads"):
        assert getattr(hf, key) == shapes[key], key
    assert hf.num_hidden_layers == 2
