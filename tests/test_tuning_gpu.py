"""Options that are off by default, against the same references as the
default paths' tests: GEMM K splits whose cluster size is not a power of two
(the reduction deals the tile's sixteen 8-feature groups unevenly over the
ranks), the L2 prefetch of the weight stream (kvb_gemm_set_l2_prefetch), the
tcgen05 GEMM backend inside the model, pipelined decode
(ModelRunner.run_async with one step in flight, and the engine's
DecodePipeline) and programmatic dependent launch (kvb_set_pdl)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from kavor_b200 import _kernels as K_
    from kavor_b200 import _lib

    _lib.load()
    _lib.device_error(clear=True)
    yield
    K_.gemm_set_l2_prefetch(0)
    assert _lib.device_error(clear=True) == 0


def _inputs(M, N, K, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("M,N,K,splits", [
    (256, 6144, 4096, 3), (64, 4096, 4096, 5), (16, 4096, 12288, 6), (256, 4096, 4096, 7), (1, 768, 4096, 10),
    (100, 1000, 1536, 3),
])
def test_gemm_non_power_of_two_cluster_split(M, N, K, splits):
    from kavor_b200 import _kernels as K_

    assert K_.gemm_plan(M, N, K, splits)["splits"] == splits
    x, w = _inputs(M, N, K)
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm(x, w, out=y, splits=splits)
    torch.testing.assert_close(y.float(), x.float() @ w.float().t(), atol=1e-2, rtol=1e-2)
    assert torch.equal(y, K_.gemm(x, w, splits=splits))  # fixed summation order


@pytest.mark.parametrize("splits", [3, 6])
def test_gated_gemm_non_power_of_two_cluster_split(splits):
    from kavor_b200 import _kernels as K_

    M, inter, K = 64, 1536, 4096
    x, w = _inputs(M, 2 * inter, K, seed=3)
    out = torch.full((M, inter), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm_silu(x, w, out=out, splits=splits)
    ref32 = x.float() @ w.float().t()
    g, u = ref32[:, :inter].to(torch.bfloat16).float(), ref32[:, inter:].to(torch.bfloat16).float()
    torch.testing.assert_close(out.float(), torch.nn.functional.silu(g) * u, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("ksteps", [2, 8, 64])
def test_gemm_l2_prefetch_leaves_results_unchanged(ksteps):
    """The prefetch only moves weight bytes into L2 early: bit-identical
    outputs, persistent and cluster schedules, plain and gated."""
    from kavor_b200 import _kernels as K_

    cases = [(256, 6144, 4096, 0, False), (7, 768, 4096, 1, False), (64, 4096, 12288, 4, False),
             (256, 3072, 4096, 0, True)]
    for M, N, K, splits, gated in cases:
        x, w = _inputs(M, (2 if gated else 1) * N, K, seed=5)
        fn = K_.gemm_silu if gated else K_.gemm
        K_.gemm_set_l2_prefetch(0)
        ref = fn(x, w, splits=splits)
        K_.gemm_set_l2_prefetch(ksteps)
        assert torch.equal(fn(x, w, splits=splits), ref), (M, N, K, splits, gated)


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    from kavor_b200.config import write_model_dir

    return write_model_dir(str(tmp_path_factory.mktemp("tiny")), "Qwen3-0.6B", num_hidden_layers=2,
                           vocab_size=4096, max_position_embeddings=4096)


def _runner(tiny_dir, **kw):
    import torch.distributed as dist

    from kavor_b200.config import Config
    from kavor_b200.engine.model_runner import ModelRunner

    if not dist.is_initialized():
        dist.init_process_group("nccl", "tcp://127.0.0.1:29565", world_size=1, rank=0,
                                device_id=torch.device("cuda", 0))
    cfg = Config(tiny_dir, load_format="dummy", seed=3, max_model_len=2048, max_num_seqs=16,
                 max_num_batched_tokens=2048, num_kvcache_blocks=64, **kw)
    return ModelRunner(cfg, 0, None)


def _greedy_decode(runner, pipelined, steps=9):
    from kavor_b200.engine.block_manager import BlockManager
    from kavor_b200.engine.model_runner import advance_decode
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    Sequence.block_size = 256
    prompts = [[(5 * i + 11 * j) % 4000 + 1 for j in range(n)] for i, n in enumerate((300, 17, 255, 1))]
    seqs = [Sequence(p, SamplingParams(max_tokens=64)) for p in prompts]
    bm = BlockManager(runner.config.num_kvcache_blocks, 256)
    for s in seqs:
        s.temperature = 0.0
        bm.allocate_prefill(s, 0)
        s.num_scheduled_tokens = s.num_tokens
    for s, t in zip(seqs, runner.run(seqs, True)):
        s.num_cached_tokens, s.num_scheduled_tokens = s.num_tokens, 0
        s.append_token(t)
        s.is_prefill = False
    advance_decode(runner, seqs, bm, steps, pipelined=pipelined)
    return [s.token_ids for s in seqs]


def test_pipelined_decode_gives_the_synchronous_tokens(tiny_dir):
    """Greedy decode through run_async (inputs chained on the device, one step
    in flight) produces exactly the tokens of the synchronous run(); the 255-
    token prompt crosses a block boundary during the steps."""
    runner = _runner(tiny_dir)
    try:
        sync = _greedy_decode(runner, False)
        piped = _greedy_decode(runner, True)
    finally:
        runner.exit()
    assert piped == sync


@pytest.mark.parametrize("prefetch", [0, 8])
def test_tcgen05_gemm_backend_replays_reference_greedy(prefetch):
    """The tiny Qwen3 with every projection on kvb_gemm_bf16 (the MLP's gate-up
    + SiLU in kvb_gemm_silu_bf16), teacher-forced on the reference model's
    prefill + 8 greedy decode steps: logits cosine >= 0.999 at every step and
    the greedy token wherever the reference's top two logits are more than
    two bf16 ulps apart; the L2 prefetch of the weights changes nothing."""
    import cases
    from conftest import GOLDEN

    from kavor_b200 import _kernels as K_
    from kavor_b200.layers.linear import set_gemm_backend
    from kavor_b200.models import AutoModelForCausalLM, _assign
    from kavor_b200.utils.context import reset_context, set_context

    dev = torch.device("cuda", 0)
    cfg = cases.hf_config(cases.TINY)
    torch.set_default_dtype(torch.bfloat16)
    torch.set_default_device(dev)
    try:
        model = AutoModelForCausalLM.model_class(cfg)(cfg)
    finally:
        torch.set_default_device("cpu")
        torch.set_default_dtype(torch.float32)
    loaded = set()
    for name, t in cases.checkpoint(cases.TINY, seed=5).items():
        _assign(model, name, t.to(dev), model.packed_modules_mapping, loaded)
    for lyr in model.model.layers:
        pool = torch.zeros(8, 2, 256, 2, 128, dtype=torch.bfloat16, device=dev)
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]

    def step(b):
        b = {k: v.to(dev) if isinstance(v, torch.Tensor) else v for k, v in b.items()}
        if b["is_prefill"]:
            n = int((b["cu_seqlens"][1:] - b["cu_seqlens"][:-1]).max())
            set_context(True, b["cu_seqlens"], b["cu_seqlens"], n, n, b["slot_mapping"])
        else:
            set_context(False, slot_mapping=b["slot_mapping"], context_lens=b["context_lens"],
                        block_tables=b["block_tables"])
        try:
            with torch.inference_mode():
                return model.compute_logits(model(b["input_ids"], b["positions"]))
        finally:
            reset_context()

    set_gemm_backend("tcgen05")
    K_.gemm_set_l2_prefetch(prefetch)
    try:
        gold = torch.load(GOLDEN / "tiny_model_golden.pt", weights_only=False)
        checked = sum(cases.check_greedy_step(logits, rec) for logits, rec in cases.replay(gold, step))
    finally:
        set_gemm_backend("auto")
        K_.gemm_set_l2_prefetch(0)
    assert checked >= 13


@pytest.mark.parametrize("gemm", ["cublas", "tcgen05"])
def test_programmatic_dependent_launch_changes_no_result(tiny_dir, gemm):
    """With every kernel launched as a programmatic dependent (kvb_set_pdl)
    inside and outside the captured decode graphs, greedy decoding gives the
    same tokens as plain stream-ordered launches: each kernel waits for the
    one before it before reading its output (the package's GEMM requests its
    first weight tiles, which no kernel writes, before that wait)."""
    from kavor_b200 import _kernels as K_
    from kavor_b200.layers.linear import set_gemm_backend

    runs = []
    for pdl in (False, True):
        runner = _runner(tiny_dir, pdl=pdl, gemm_backend=gemm)
        try:
            runs.append(_greedy_decode(runner, False))
        finally:
            runner.exit()
            K_.set_pdl(False)
            set_gemm_backend("auto")
    assert runs[0] == runs[1]


def test_async_decode_engine_gives_the_same_generations(tiny_dir):
    """LLM.generate with one decode step in flight (Config.async_decode)
    returns the generations of the step-at-a-time engine: sampled at
    temperature 0.6 with ignore_eos, the steps see the same batches in the
    same order and the same sampler seeds."""
    import torch.distributed as dist

    from kavor_b200 import LLM, SamplingParams

    prompts = [[(3 * j + i) % 4000 + 1 for j in range(n)] for i, n in enumerate((300, 17, 700, 1, 64))]
    params = [SamplingParams(temperature=0.6, max_tokens=m, ignore_eos=True) for m in (9, 30, 4, 17, 12)]
    outs = []
    for async_decode in (False, True):
        if dist.is_initialized():
            dist.destroy_process_group()
        llm = LLM(tiny_dir, load_format="dummy", seed=1, max_model_len=2048, max_num_seqs=8,
                  max_num_batched_tokens=512, num_kvcache_blocks=32, rdzv_port=29577 + int(async_decode),
                  async_decode=async_decode)
        try:
            outs.append([o["token_ids"] for o in llm.generate(prompts, params, use_tqdm=False)])
        finally:
            llm.exit()
    assert [len(o) for o in outs[1]] == [9, 30, 4, 17, 12]
    assert outs[0] == outs[1]
