"""The product's model classes on the CPU, kernels swapped for the oracle.

Qwen3, Mistral and ERNIE 4.5 (``kavor_b200.models``) are built from their
configs through the registry, loaded through the dummy checkpoint loader and
the TP weight loaders, and run the reference's greedy fixtures
(tests/golden/make_golden.py) teacher-forced. Every kernel wrapper of
``kavor_b200._kernels`` that the forward calls is replaced, for this test
only, by its oracle restatement, so what is checked is the Python wiring
above the C ABI: the attention flags of each family (q/k norm, bias,
interleaved RoPE), the residual wiring, parameter names and sharding, the
tied/untied LM head. The kernels themselves are checked against the same
fixtures on the GPU (test_model_gpu.py)."""
import pytest
import torch

import cases
from conftest import GOLDEN
from oracle import ops


def _qknorm_rope_store(qkv, hq, hkv, hd, q_weight, k_weight, eps, positions, cos_sin, interleaved,
                       k_cache, v_cache, slot_mapping):
    T = qkv.shape[0]
    q = qkv[:, :hq * hd].view(T, hq, hd)
    k = qkv[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd)
    v = qkv[:, (hq + hkv) * hd:].view(T, hkv, hd)
    qn = ops.rmsnorm(q, q_weight, eps) if q_weight is not None else q
    kn = ops.rmsnorm(k, k_weight, eps) if k_weight is not None else k
    q.copy_(ops.rope(qn, positions, cos_sin, interleaved))
    k.copy_(ops.rope(kn, positions, cos_sin, interleaved))
    if k_cache is not None:
        ops.store_kvcache(k, v, k_cache, v_cache, slot_mapping)


def _add_rmsnorm(x, residual, weight, eps, out=None):
    y, r = ops.add_rmsnorm(x, residual, weight, eps)
    residual.copy_(r)
    return y, residual


def _embedding(ids, weight, start, end, vocab, out=None):
    y = ops.embedding(ids.reshape(-1), weight, start, end)
    return y if out is None else out.copy_(y)


def _prefill(q, k, v, cu_q, cu_k, max_q, scale, block_tables=None, out=None, tensor_cores=True):
    return ops.varlen_prefill_attention(q, k, v, cu_q, cu_k, scale, block_tables)


def _decode(q, k_cache, v_cache, block_tables, context_lens, scale, out=None, num_splits=0, workspace=None):
    return ops.paged_decode_attention(q, k_cache, v_cache, block_tables, context_lens, scale)


# kernel wrapper name -> its oracle restatement (also used by the gloo TP tests)
ORACLE_KERNELS = (("qknorm_rope_store", _qknorm_rope_store), ("add_rmsnorm", _add_rmsnorm),
                  ("rmsnorm", lambda x, w, eps, out=None: ops.rmsnorm(x, w, eps)),
                  ("silu_mul", lambda x, out=None: ops.silu_mul(x)), ("embedding", _embedding),
                  ("prefill_attention", _prefill), ("paged_decode_attention", _decode))


@pytest.fixture
def oracle_kernels(monkeypatch):
    from kavor_b200 import _kernels as K

    for name, fn in ORACLE_KERNELS:
        monkeypatch.setattr(K, name, fn)


def _model(cfg):
    from kavor_b200.models import AutoModelForCausalLM

    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        model = AutoModelForCausalLM.model_class(cfg)(cfg)
    finally:
        torch.set_default_dtype(prev)
    AutoModelForCausalLM.load_weight(model, cfg, load_format="dummy", seed=5)  # the fixtures' checkpoint
    return model


CASES = [("qwen3", "tiny_model_golden.pt")] + [(f, f"{f}_tiny_golden.pt") for f in cases.FAMILIES]


@pytest.fixture(params=["auto", "cublas", "tcgen05", "tcgen05_pair"])
def gemm_backend(request, monkeypatch):
    """Every GEMM backend of linear(): torch's F.linear, or the package's
    kernel entry points (replaced here by the oracle's linear, with the gate-up
    + SiLU fusion of the MLP as silu_mul(linear))."""
    from kavor_b200 import _kernels as K
    from kavor_b200.layers import linear as L

    def gemm(x, w, out=None, splits=0):
        return ops.linear(x, w) if out is None else out.copy_(ops.linear(x, w))

    if request.param != "cublas":
        monkeypatch.setattr(K, "gemm", gemm)
        monkeypatch.setattr(K, "gemm_pair", gemm)
        monkeypatch.setattr(K, "gemm_sk", gemm)
        monkeypatch.setattr(K, "gemm_silu", lambda x, w, out=None, splits=0: ops.silu_mul(ops.linear(x, w)))
        monkeypatch.setattr(K, "gemm_pair_silu", lambda x, w, out=None: ops.silu_mul(ops.linear(x, w)))
        monkeypatch.setattr(K, "gemm_sk_silu", lambda x, w, out=None: ops.silu_mul(ops.linear(x, w)))
    L.set_gemm_backend(request.param)
    yield request.param
    L.set_gemm_backend("auto")


@pytest.mark.parametrize("family,fixture", CASES, ids=[c[0] for c in CASES])
def test_model_classes_replay_reference_greedy(oracle_kernels, gemm_backend, family, fixture):
    cfg = cases.hf_config(cases.TINY) if family == "qwen3" else cases.family_config(family)
    model = _model(cfg)
    for lyr in model.model.layers:
        pool = torch.zeros(8, 2, 256, cfg.num_key_value_heads, 128, dtype=torch.bfloat16)
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]

    gold = torch.load(GOLDEN / fixture, weights_only=False)
    # with the oracle's kernels the logits differ from the reference's only by
    # matmul summation order (cosine > 0.99998 here), so the bound is tighter
    # than the GPU's 0.999: a wrong rope theta or rotation stays above 0.998
    checked = sum(cases.check_greedy_step(logits, rec, min_cos=0.9999)
                  for logits, rec in cases.replay(gold, lambda b: cases.model_step(model, b)))
    assert checked >= 13  # at least half of the 27 tokens


def test_model_classes_prefix_cache_prefill(oracle_kernels):
    """The prefill of a prompt whose first block is already cached: the
    attention layer reads K/V from the paged cache through the block table
    (cu_seqlens_k > cu_seqlens_q), as ModelRunner.prepare_prefill sets it up."""
    cfg = cases.hf_config(cases.TINY)
    model = _model(cfg)
    for lyr in model.model.layers:
        pool = torch.zeros(8, 2, 256, cfg.num_key_value_heads, 128, dtype=torch.bfloat16)
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]
    gold = torch.load(GOLDEN / "prefix_cache_golden.pt", weights_only=False)
    checked = sum(cases.check_greedy_step(logits, rec, min_cos=0.9999)
                  for logits, rec in cases.replay_prefix_cache(gold, lambda b: cases.model_step(model, b)))
    assert checked >= 9  # of 10


def test_gemm_backend_names():
    from kavor_b200.layers import linear as L

    with pytest.raises(ValueError, match="unknown GEMM backend"):
        L.set_gemm_backend("triton")
    assert L.gemm_backend() == "auto"


def test_auto_gemm_dispatch_rule():
    """The default backend puts the full-vocabulary LM head of Qwen3-8B on the
    stream-K kernel at decode batches and every decoder-layer projection (and
    the TP=8 vocabulary shard, and prefill batches) on F.linear."""
    from kavor_b200.layers import linear as L

    assert L.auto_uses_stream_k(256, 151936, 4096) and L.auto_uses_stream_k(1, 151936, 4096)
    assert not L.auto_uses_stream_k(257, 151936, 4096)
    for N, K in ((6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288), (18992, 4096), (151936, 1024)):
        assert not L.auto_uses_stream_k(256, N, K), (N, K)


def test_family_attention_flags():
    """Per family: which optional attention tensors exist and which RoPE runs
    (qwen3.py:71-73, mistral.py:37-82, ernie4_5.py:61-88)."""
    from kavor_b200.models import AutoModelForCausalLM

    expect = {"qwen3": (True, False, False), "mistral": (False, False, False), "ernie4_5": (False, True, True)}
    for family, (qk_norm, bias, interleaved) in expect.items():
        cfg = cases.hf_config(cases.TINY) if family == "qwen3" else cases.family_config(family)
        attn = AutoModelForCausalLM.model_class(cfg)(cfg).model.layers[0].self_attn
        assert attn.qk_norm == qk_norm and hasattr(attn, "q_norm") == qk_norm, family
        assert (attn.qkv_proj.bias is not None) == bias, family
        assert attn.rotary_emb.interleaved == interleaved, family
