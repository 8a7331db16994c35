"""Model-level parity on the GPU: the Qwen3 layer/model built from kavor_b200
layers against the reference's own outputs (tests/golden), and the engine
(ModelRunner / LLM.generate) end to end."""
import pytest
import torch

import cases
from conftest import GOLDEN

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")


def _build(fn):
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    torch.set_default_device(DEV)
    try:
        return fn()
    finally:
        torch.set_default_device("cpu")
        torch.set_default_dtype(prev)


def _load(module, tensors, packed):
    from kavor_b200.models import _assign

    loaded = set()
    for name, t in tensors.items():
        _assign(module, name, t.to(DEV), packed, loaded)


@pytest.fixture
def gemm_backend(request):
    """Run the test with the projections on the named GEMM backend."""
    from kavor_b200.layers.linear import set_gemm_backend

    set_gemm_backend(request.param)
    try:
        yield request.param
    finally:
        set_gemm_backend("auto")


BACKENDS = ["cublas", "tcgen05", "tcgen05_pair"]


@pytest.mark.parametrize("gemm_backend", BACKENDS, indirect=True)
def test_config1_decoder_layer_matches_reference(gemm_backend):
    """One Qwen3-0.6B layer, one decode step, B=16, vs the reference layer's
    output: max-abs 2e-2 / rel 1e-2 (the per-layer parity bound), with the
    projections on every GEMM backend."""
    _replay_layer_golden(cases.config1_layer_case(0), "layer_golden.pt")


def _assert_close_tail(actual, expected, frac=1e-3, atol=2e-2, rtol=1e-2):
    """The per-layer bound |a - b| <= atol + rtol |b| for all but `frac` of the
    elements, and twice that bound for every element."""
    a, b = actual.float().cpu(), expected.float().cpu()
    d, bound = (a - b).abs(), atol + rtol * b.abs()
    over = (d > bound).float().mean().item()
    assert over <= frac, f"{over:.2e} of the outputs beyond the bound (max |diff| {d.max().item():.4f})"
    assert bool((d <= 2 * bound).all()), f"max excess over twice the bound {(d - 2 * bound).max().item():.4f}"


@pytest.mark.parametrize("gemm_backend", BACKENDS, indirect=True)
def test_8b_decoder_layer_matches_reference(gemm_backend):
    """One Qwen3-8B layer (the headline model's shapes: hidden 4096, 32 q / 8
    kv heads, intermediate 12288), one decode step of 8 sequences at context
    1024, first layer (no residual) and a later one.

    Two references: the reference's arithmetic run on this GPU
    (tests/reference_gpu: cuBLAS projections and the flash-attn decode call,
    as the reference runs them), and the reference layer's CPU fixture. The
    residual must be within max-abs 2e-2 / rel 1e-2 at every element; the
    output within that bound for all but 0.1 % of the elements and within
    twice it everywhere. Any two implementations of this layer that sum in
    different orders (the CPU's fp32 GEMMs, flash-attn's and this package's
    attention) round a few of the 12288 bf16 intermediates per row to the
    other side; over K = 12288 the down projection's outputs (std 2.3) then
    move by about 0.006, and among 32768 outputs a handful reach 0.03 (seen
    here: 3 outputs against either reference) — the spread between the
    reference's own eager and compiled SiluAndMul forms."""
    import reference_gpu

    fa = reference_gpu.flash_attn_or_none()
    case = cases.config3_layer_case(0)
    gold = torch.load(GOLDEN / "layer_8b_golden.pt", weights_only=False)
    for variant, res, (h, r) in _run_layer(case):
        torch.testing.assert_close(r.float().cpu(), gold[variant]["residual"].float(), atol=2e-2, rtol=1e-2)
        _assert_close_tail(h, gold[variant]["hidden"])
        if fa is None:
            continue
        pool = case["pool"].to(DEV)
        with torch.inference_mode():
            rh, rr = reference_gpu.decode_layer(
                fa, case["layer"], case["shape"], case["hidden"].to(DEV), None if res is None else res.to(DEV),
                case["positions"].to(DEV), case["slot_mapping"].to(DEV), case["context_lens"].to(DEV),
                case["block_tables"].to(DEV), pool[:, 0], pool[:, 1])
        torch.testing.assert_close(r.float(), rr.float(), atol=2e-2, rtol=1e-2)
        _assert_close_tail(h, rh)


def _run_layer(case):
    """Yields (variant, residual input, (hidden, residual)) of the product's
    decoder layer for the first-layer and later-layer wiring."""
    from kavor_b200.models.qwen3 import Qwen3DecoderLayer, Qwen3ForCausalLM
    from kavor_b200.utils.context import reset_context, set_context

    layer = _build(lambda: Qwen3DecoderLayer(cases.hf_config(case["shape"])))
    _load(layer, case["layer"], Qwen3ForCausalLM.packed_modules_mapping)
    for variant, res in (("first", None), ("later", case["residual"])):
        pool = case["pool"].to(DEV)
        layer.self_attn.attn.k_cache = [pool[:, 0]]
        layer.self_attn.attn.v_cache = [pool[:, 1]]
        set_context(False, slot_mapping=case["slot_mapping"].to(DEV), context_lens=case["context_lens"].to(DEV),
                    block_tables=case["block_tables"].to(DEV))
        try:
            with torch.inference_mode():
                out = layer(case["positions"].to(DEV), case["hidden"].to(DEV), None if res is None else res.to(DEV))
        finally:
            reset_context()
        yield variant, res, out


def _replay_layer_golden(case, fixture):
    gold = torch.load(GOLDEN / fixture, weights_only=False)
    for variant, _, (h, r) in _run_layer(case):
        torch.testing.assert_close(r.float().cpu(), gold[variant]["residual"].float(), atol=2e-2, rtol=1e-2)
        torch.testing.assert_close(h.float().cpu(), gold[variant]["hidden"].float(), atol=2e-2, rtol=1e-2)


def test_tiny_model_greedy_tokens_and_logits_match_reference():
    """Prefill + 8 decode steps of a 2-layer Qwen3: greedy tokens equal the
    reference's, logits cosine >= 0.999 at every step."""
    from kavor_b200.models import AutoModelForCausalLM
    from kavor_b200.utils.context import reset_context, set_context

    gold = torch.load(GOLDEN / "tiny_model_golden.pt", weights_only=False)
    cfg = cases.hf_config(cases.TINY)
    model = _build(lambda: AutoModelForCausalLM.model_class(cfg)(cfg))
    _load(model, cases.checkpoint(cases.TINY, seed=5), model.packed_modules_mapping)
    pools = [torch.zeros(8, 2, 256, 2, 128, dtype=torch.bfloat16, device=DEV) for _ in range(2)]
    for lyr, pool in zip(model.model.layers, pools):
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]
    seqs = [list(p) for p in gold["prompts"]]
    tables = gold["tables"]
    i32 = dict(dtype=torch.int32, device=DEV)
    with torch.inference_mode():
        ids = torch.tensor([t for s in seqs for t in s], device=DEV)
        pos = torch.tensor([i for s in seqs for i in range(len(s))], device=DEV)
        cu = torch.tensor([0] + torch.tensor([len(s) for s in seqs]).cumsum(0).tolist(), **i32)
        slots = torch.tensor([tables[b][0] * 256 + i for b, s in enumerate(seqs) for i in range(len(s))], **i32)
        set_context(True, cu, cu, max(map(len, seqs)), max(map(len, seqs)), slots)
        logits = model.compute_logits(model(ids, pos))
        reset_context()
        for step in gold["steps"]:
            cos = torch.nn.functional.cosine_similarity(logits.float().cpu(), step["logits"].float(), dim=-1)
            assert cos.min().item() >= 0.999
            tok = logits.float().argmax(-1).tolist()
            assert tok == step["tokens"]
            for b, t in enumerate(tok):
                seqs[b].append(t)
            set_context(False, slot_mapping=torch.tensor([tables[b][0] * 256 + len(s) - 1 for b, s in enumerate(seqs)], **i32),
                        context_lens=torch.tensor([len(s) for s in seqs], **i32),
                        block_tables=torch.tensor(tables, **i32))
            logits = model.compute_logits(model(torch.tensor([s[-1] for s in seqs], device=DEV),
                                                torch.tensor([len(s) - 1 for s in seqs], device=DEV)))
            reset_context()


def _tiny_model():
    from kavor_b200.models import AutoModelForCausalLM

    cfg = cases.hf_config(cases.TINY)
    model = _build(lambda: AutoModelForCausalLM.model_class(cfg)(cfg))
    _load(model, cases.checkpoint(cases.TINY, seed=5), model.packed_modules_mapping)
    for lyr in model.model.layers:
        pool = torch.zeros(8, 2, 256, 2, 128, dtype=torch.bfloat16, device=DEV)
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]
    return model


@pytest.mark.parametrize("gemm_backend", BACKENDS, indirect=True)
def test_tiny_model_32_greedy_tokens_match_reference(gemm_backend):
    """32 greedy tokens (prefill + 31 decode steps) of the reference's 2-layer
    Qwen3, teacher-forced on the reference's tokens: at every step the
    product's argmax equals the reference's token wherever the reference's two
    largest logits are more than two bf16 ulps apart, and its logits have
    cosine >= 0.999 against the oracle's (pinned to the reference model on the
    CPU) for the same inputs; every GEMM backend."""
    from oracle import model as omodel

    gold = torch.load(GOLDEN / "tiny_model_golden_32.pt", weights_only=False)
    assert len(gold["steps"]) == 32
    model = _tiny_model()
    shape = omodel.Shape(hidden=512, inter=1024, layers=2, hq=4, hkv=2, vocab=4096)
    p = cases.checkpoint(cases.TINY, seed=5)
    kv = [(torch.zeros(8, 256, 2, 128, dtype=torch.bfloat16), torch.zeros(8, 256, 2, 128, dtype=torch.bfloat16))
          for _ in range(2)]

    def step(b):
        logits = cases.model_step(model, b, DEV).float().cpu()
        batch = (omodel.Batch(True, b["positions"], b["slot_mapping"], b["cu_seqlens"], b["cu_seqlens"])
                 if b["is_prefill"] else
                 omodel.Batch(False, b["positions"], b["slot_mapping"], context_lens=b["context_lens"],
                              block_tables=b["block_tables"]))
        ref = omodel.forward(p, b["input_ids"], batch, kv, shape)[1].float()
        cos = torch.nn.functional.cosine_similarity(logits, ref, dim=-1)
        assert cos.min().item() >= 0.999, cos
        return logits

    checked = sum(cases.check_greedy_step(logits, rec) for logits, rec in cases.replay(gold, step))
    assert checked >= 84  # of 96 (3 sequences x 32 tokens)


@pytest.mark.parametrize("family", cases.FAMILIES)
def test_family_model_replays_reference_greedy(family):
    """Tiny Mistral (no q/k norm, no bias) and ERNIE 4.5 (q/k/v bias,
    interleaved RoPE) on the kernels, teacher-forced on the reference model's
    prefill + 8 greedy decode steps: logits cosine >= 0.999 at every step and
    the greedy token wherever the reference's top two logits are more than two
    bf16 ulps apart."""
    from kavor_b200.models import AutoModelForCausalLM

    cfg = cases.family_config(family)
    model = _build(lambda: AutoModelForCausalLM.model_class(cfg)(cfg))
    _load(model, cases.family_checkpoint(family, seed=5), model.packed_modules_mapping)
    for lyr in model.model.layers:
        pool = torch.zeros(8, 2, 256, cfg.num_key_value_heads, 128, dtype=torch.bfloat16, device=DEV)
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]

    gold = torch.load(GOLDEN / f"{family}_tiny_golden.pt", weights_only=False)
    checked = sum(cases.check_greedy_step(logits, rec)
                  for logits, rec in cases.replay(gold, lambda b: cases.model_step(model, b, DEV)))
    assert checked >= 13  # at least half of the 27 tokens


def test_prefix_cache_prefill_replays_reference_greedy():
    """A prompt whose first 256-token block is already in the cache prefills
    only its 40 new tokens: the paged prefill attention reads the cached block
    through the block table (cu_seqlens_k 296 > cu_seqlens_q 40); then both
    prompts decode 4 steps. Logits cosine >= 0.999 and the reference model's
    greedy token at every step."""
    from kavor_b200.models import AutoModelForCausalLM

    cfg = cases.hf_config(cases.TINY)
    model = _build(lambda: AutoModelForCausalLM.model_class(cfg)(cfg))
    _load(model, cases.checkpoint(cases.TINY, seed=5), model.packed_modules_mapping)
    for lyr in model.model.layers:
        pool = torch.zeros(8, 2, 256, 2, 128, dtype=torch.bfloat16, device=DEV)
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]
    gold = torch.load(GOLDEN / "prefix_cache_golden.pt", weights_only=False)
    checked = sum(cases.check_greedy_step(logits, rec)
                  for logits, rec in cases.replay_prefix_cache(gold, lambda b: cases.model_step(model, b, DEV)))
    assert checked >= 9  # of 10


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    from kavor_b200.config import write_model_dir

    return write_model_dir(str(tmp_path_factory.mktemp("tiny")), "Qwen3-0.6B", num_hidden_layers=2,
                           vocab_size=4096, max_position_embeddings=4096)


def _runner(tiny_dir, eager: bool):
    import torch.distributed as dist

    from kavor_b200.config import Config
    from kavor_b200.engine.model_runner import ModelRunner

    if not dist.is_initialized():
        dist.init_process_group("nccl", "tcp://127.0.0.1:29561", world_size=1, rank=0, device_id=DEV)
    cfg = Config(tiny_dir, load_format="dummy", seed=3, enforce_eager=eager, max_model_len=2048,
                 max_num_seqs=16, max_num_batched_tokens=2048, num_kvcache_blocks=64)
    return ModelRunner(cfg, 0, None)


def _greedy_seqs(prompts):
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    seqs = [Sequence(p, SamplingParams(max_tokens=8)) for p in prompts]
    for s in seqs:
        s.temperature = 0.0  # engine-internal greedy (SamplingParams forbids 0)
    return seqs


def test_model_runner_graph_decode_equals_eager(tiny_dir):
    """ModelRunner prefill + decode steps: CUDA-graph replay gives the same
    greedy tokens as the eager path."""
    from kavor_b200.engine.block_manager import BlockManager
    from kavor_b200.engine.sequence import Sequence

    Sequence.block_size = 256
    prompts = [[(5 * i + 11 * j) % 4000 + 1 for j in range(n)] for i, n in enumerate((300, 17, 256, 1))]
    results = []
    for eager in (True, False):
        runner = _runner(tiny_dir, eager)
        bm = BlockManager(runner.config.num_kvcache_blocks, 256)
        seqs = _greedy_seqs(prompts)
        for s in seqs:
            bm.allocate_prefill(s, 0)
            s.num_scheduled_tokens = s.num_tokens
        toks = [runner.run(seqs, True)]
        for s, t in zip(seqs, toks[0]):
            s.num_cached_tokens, s.num_scheduled_tokens = s.num_tokens, 0
            s.append_token(t)
            s.is_prefill = False
        for _ in range(6):
            for s in seqs:
                bm.may_append_block(s)
            out = runner.run(seqs, False)
            toks.append(out)
            for s, t in zip(seqs, out):
                s.num_cached_tokens += 1
                s.append_token(t)
        results.append(toks)
        runner.exit()
    assert results[0] == results[1]


def test_llm_generate_prefix_cache_and_chunking(tiny_dir):
    """LLM.generate end to end: a repeated long prompt hits the prefix cache,
    a prompt longer than the token budget is chunked, every request finishes
    with max_tokens tokens."""
    import torch.distributed as dist

    from kavor_b200 import LLM, SamplingParams

    if dist.is_initialized():
        dist.destroy_process_group()
    llm = LLM(tiny_dir, load_format="dummy", seed=1, max_model_len=2048, max_num_seqs=8,
              max_num_batched_tokens=512, num_kvcache_blocks=32, rdzv_port=29573)
    try:
        long = [(3 * j) % 4000 + 1 for j in range(700)]
        out = llm.generate([long, [1, 2, 3]], SamplingParams(temperature=0.6, max_tokens=5, ignore_eos=True),
                           use_tqdm=False)
        assert [len(o["token_ids"]) for o in out] == [5, 5]
        before = llm.scheduler.block_manager.prefix_cache_hit_tokens
        out = llm.generate([long], SamplingParams(temperature=0.6, max_tokens=4, ignore_eos=True), use_tqdm=False)
        assert len(out[0]["token_ids"]) == 4
        assert llm.scheduler.block_manager.prefix_cache_hit_tokens >= before + 512
    finally:
        llm.exit()
