"""Engine configuration (drop-in for kavor/config.py:16-53, text models).

Extra fields over the reference: ``load_format`` ("auto" reads the checkpoint
in ``model``, "dummy" draws a seeded random checkpoint of the same shapes),
``seed`` for that draw, ``enable_prefix_caching`` (the reference always
caches prefixes), ``graph_batch_sizes`` (the decode batch buckets captured
as CUDA graphs; default: the reference's 1, 2, 4, 8 and multiples of 16),
``fused_allreduce``, ``gemm_backend`` / ``gemm_l2_prefetch`` (which GEMM
the projections use, and its L2 prefetch distance), ``pdl`` (programmatic
dependent launch of the package's kernels), ``async_decode`` (the engine
keeps one decode step in flight) and ``decode_microbatches`` /
``decode_microbatch_min_bs`` (TP > 1: a decode batch of at least that many
sequences runs as two halves on two streams, each half's all-reduces and
GEMMs beside the other half's attention).
"""
from __future__ import annotations

import json
import os
import socket
from dataclasses import dataclass
from typing import Any


def free_port() -> int:
    if env := os.environ.get("KAVOR_RDZV_PORT"):
        return int(env)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def load_hf_config(model_dir: str):
    """Text config of a model directory (transformers' own parser)."""
    from transformers import AutoConfig

    return AutoConfig.from_pretrained(model_dir, trust_remote_code=False)


@dataclass(slots=True)
class Config:
    model: str
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.9
    tensor_parallel_size: int = 1
    enforce_eager: bool = False
    profile: bool = False
    trust_remote_code: bool = False
    hf_config: Any = None
    eos: int = -1
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    rdzv_port: int = -1
    load_format: str = "auto"
    seed: int = 0
    enable_prefix_caching: bool = True
    graph_batch_sizes: tuple[int, ...] | None = None  # decode buckets to capture (None: 1,2,4,8,16,32,...)
    fused_allreduce: bool = True  # TP > 1: NVLink all-reduce fused with add+RMSNorm (False: NCCL + separate norm)
    gemm_backend: str = "auto"  # projections: "auto" (stream-K kernel where it measured faster, F.linear elsewhere), "cublas" (F.linear), "tcgen05" (the package's kernels, fused gate-up+SiLU),
    #                               "tcgen05_pair" (kvb_gemm_pair_bf16)
    gemm_l2_prefetch: int = 0     # tcgen05 GEMM: weight K-steps prefetched into L2 ahead of the loads (0 = off)
    pdl: bool = False             # programmatic dependent launch of the package's kernels (kvb_set_pdl)
    async_decode: bool = False    # LLM.generate: one decode step in flight (engine.pipeline.DecodePipeline)
    decode_microbatches: int = 1  # TP > 1 with the fused all-reduce: 2 = decode as two halves on two streams
    decode_microbatch_min_bs: int = 64  # smallest decode batch that is split (smaller ones run whole)

    def __post_init__(self):
        if not os.path.isdir(self.model):
            raise RuntimeError(f"Model not found: {self.model}")
        assert self.kvcache_block_size % 256 == 0, "kvcache_block_size must be a multiple of 256"
        assert 1 <= self.tensor_parallel_size <= 8
        assert self.load_format in ("auto", "dummy")
        assert self.gemm_backend in ("auto", "cublas", "tcgen05", "tcgen05_pair"), "unknown gemm_backend"
        assert 0 <= self.gemm_l2_prefetch <= 64
        assert self.decode_microbatches in (1, 2), "decode_microbatches must be 1 or 2"
        assert self.decode_microbatch_min_bs >= 2
        self.rdzv_port = self.rdzv_port if self.rdzv_port > 0 else free_port()
        if self.hf_config is None:
            self.hf_config = load_hf_config(self.model)
        self.max_model_len = min(self.max_model_len, self.hf_config.max_position_embeddings)

    @property
    def text_config(self):
        return self.hf_config


# Shapes of the Qwen3 dense models used by the benchmarks (config.json fields).
QWEN3_PRESETS: dict[str, dict] = {
    "Qwen3-0.6B": dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28, num_attention_heads=16,
                       num_key_value_heads=8, head_dim=128, tie_word_embeddings=True),
    "Qwen3-8B": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, head_dim=128, tie_word_embeddings=False),
    "Qwen3-32B": dict(hidden_size=5120, intermediate_size=25600, num_hidden_layers=64, num_attention_heads=64,
                      num_key_value_heads=8, head_dim=128, tie_word_embeddings=False),
}

# The other dense families the model registry serves, one published size each.
FAMILY_PRESETS: dict[str, dict] = {
    "Mistral-7B-v0.3": dict(architectures=["MistralForCausalLM"], model_type="mistral", vocab_size=32768,
                            hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
                            num_key_value_heads=8, head_dim=128, max_position_embeddings=32768, rms_norm_eps=1e-5,
                            rope_theta=1000000.0, hidden_act="silu", sliding_window=None, tie_word_embeddings=False,
                            torch_dtype="bfloat16", bos_token_id=1, eos_token_id=2),
    "ERNIE-4.5-0.3B": dict(architectures=["Ernie4_5ForCausalLM"], model_type="ernie4_5", vocab_size=103424,
                           hidden_size=1024, intermediate_size=3072, num_hidden_layers=18, num_attention_heads=16,
                           num_key_value_heads=2, head_dim=128, max_position_embeddings=131072, rms_norm_eps=1e-5,
                           rope_theta=500000.0, hidden_act="silu", use_bias=False, tie_word_embeddings=True,
                           torch_dtype="bfloat16", bos_token_id=1, eos_token_id=2),
}


def write_model_dir(path: str, preset: str, **overrides) -> str:
    """Write a weight-less model directory (config.json only) for load_format='dummy'."""
    if preset in FAMILY_PRESETS:
        cfg = dict(FAMILY_PRESETS[preset])
    else:
        cfg = dict(architectures=["Qwen3ForCausalLM"], model_type="qwen3", vocab_size=151936,
                   max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1000000.0, hidden_act="silu",
                   attention_bias=False, torch_dtype="bfloat16", bos_token_id=151643, eos_token_id=151645)
        cfg.update(QWEN3_PRESETS[preset])
    cfg.update(overrides)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return path
