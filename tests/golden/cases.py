"""Seeded inputs shared by the golden-fixture generator and the tests.

Every case is rebuilt from its seed on demand (CPU generators are
deterministic for a given torch build), so the committed fixtures only hold
outputs and small metadata. Shapes follow the one-layer case and the 8B decode case:
Qwen3-0.6B / Qwen3-8B layer shapes, head_dim 128, block_size 256, context
lengths U[100, 1024] from seed 0, KV pages N(0, 1), block tables a random
permutation of the pool's blocks.
"""
from __future__ import annotations

import random

import torch

QWEN3_06B = dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28, num_attention_heads=16,
                 num_key_value_heads=8, head_dim=128, tie_word_embeddings=True)
QWEN3_8B = dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                num_key_value_heads=8, head_dim=128, tie_word_embeddings=False)
TINY = dict(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, head_dim=128, tie_word_embeddings=False, vocab_size=4096)


def hf_config(shape: dict, **over):
    from transformers import Qwen3Config

    kw = dict(vocab_size=151936, max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6,
              attention_bias=False, hidden_act="silu")
    kw.update(shape)
    kw.update(over)
    cfg = Qwen3Config(**kw)
    cfg.rope_scaling = {"rope_theta": 1e6, "rope_type": "default"}
    return cfg


# Tiny members of the other dense families (2 layers, TINY shapes, untied LM
# head: a tied head on random weights repeats the prompt's last token). Mistral:
# no q/k norm, no bias, rope theta 1e4; ERNIE 4.5: q/k/v bias, interleaved
# RoPE, theta 5e5. Both with eps 1e-5 (their published configs').
FAMILIES = ("mistral", "ernie4_5")


def prefix_cache_prompts() -> tuple[list[int], list[int]]:
    """Prompt A (300 tokens) and the 40 new tokens that follow A's first 256
    (one full block) in prompt B."""
    g = torch.Generator().manual_seed(21)
    return (torch.randint(3, 4000, (300,), generator=g).tolist(), torch.randint(3, 4000, (40,), generator=g).tolist())


def family_config(family: str):
    from transformers import Ernie4_5Config, MistralConfig

    kw = dict(TINY, max_position_embeddings=4096, rms_norm_eps=1e-5, hidden_act="silu")
    if family == "mistral":
        return MistralConfig(**kw, rope_theta=10000.0)
    if family == "ernie4_5":
        kw.update(use_bias=True)
        return Ernie4_5Config(**kw, rope_theta=500000.0)
    raise ValueError(family)


def family_checkpoint(family: str, seed: int = 0) -> dict[str, torch.Tensor]:
    """Full checkpoint of the tiny family model drawn by kavor_b200's dummy loader."""
    from kavor_b200.models import synthetic_checkpoint

    return dict(synthetic_checkpoint(family_config(family), seed, torch.device("cpu")))


def family_oracle_shape(family: str):
    from oracle import model as omodel

    cfg = family_config(family)
    theta = cfg.rope_parameters["rope_theta"]
    return omodel.Shape(hidden=cfg.hidden_size, inter=cfg.intermediate_size, layers=cfg.num_hidden_layers,
                        hq=cfg.num_attention_heads, hkv=cfg.num_key_value_heads, vocab=cfg.vocab_size,
                        eps=cfg.rms_norm_eps, rope_theta=theta, tie=False,
                        qk_norm=False, qkv_bias=family == "ernie4_5", interleaved=family == "ernie4_5",
                        separate_residual_add=family == "ernie4_5")


def checkpoint(shape: dict, seed: int = 0, layers: int | None = None) -> dict[str, torch.Tensor]:
    """Full (TP=1) checkpoint tensors drawn on the CPU by kavor_b200's dummy loader."""
    from kavor_b200.models import synthetic_checkpoint

    over = {} if layers is None else {"num_hidden_layers": layers}
    return dict(synthetic_checkpoint(hf_config(shape, **over), seed, torch.device("cpu")))


def paged_pool(num_blocks: int, block_size: int, hkv: int, hd: int, seed: int):
    """K/V caches in the reference page layout (K block then V block per page),
    filled with N(0, 1) bf16. Returns (pool, k_cache, v_cache)."""
    g = torch.Generator().manual_seed(seed)
    pool = torch.randn(num_blocks, 2, block_size, hkv, hd, generator=g).to(torch.bfloat16)
    return pool, pool[:, 0], pool[:, 1]


def decode_batch(batch: int, lo: int, hi: int, block_size: int, seed: int, spare_blocks: int = 4):
    """Context lengths U[lo, hi] (random.Random(seed)), block tables from a
    permutation of the pool (torch generator seed + 1). Returns
    (context_lens, block_tables [-1 padded], num_blocks, positions, slot_mapping)."""
    rng = random.Random(seed)
    ctx = [rng.randint(lo, hi) for _ in range(batch)]
    need = [(c + block_size - 1) // block_size for c in ctx]
    num_blocks = sum(need) + spare_blocks
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(seed + 1)).tolist()
    width = max(need)
    tables, k = [], 0
    for n in need:
        tables.append(perm[k:k + n] + [-1] * (width - n))
        k += n
    positions = [c - 1 for c in ctx]
    slots = [tables[i][(c - 1) // block_size] * block_size + (c - 1) % block_size for i, c in enumerate(ctx)]
    return (torch.tensor(ctx, dtype=torch.int32), torch.tensor(tables, dtype=torch.int32), num_blocks,
            torch.tensor(positions, dtype=torch.int64), torch.tensor(slots, dtype=torch.int32))


def config1_layer_case(seed: int = 0) -> dict:
    """The one-layer case: one Qwen3-0.6B decoder layer, one decode step, B = 16."""
    return decode_layer_case(QWEN3_06B, 16, 100, 1024, seed)


def config3_layer_case(seed: int = 0) -> dict:
    """One Qwen3-8B decoder layer (the headline model's shapes: hidden 4096,
    32 q / 8 kv heads, intermediate 12288), one decode step of 8 sequences at
    the decode-scaling case's fixed 1024-token context."""
    return decode_layer_case(QWEN3_8B, 8, 1024, 1024, seed)


def decode_layer_case(shape: dict, batch: int, lo: int, hi: int, seed: int) -> dict:
    """One decoder layer of `shape` (weights from the dummy loader), one decode
    step of `batch` sequences with contexts U[lo, hi]: hidden and residual
    rows N(0, 1), KV pages N(0, 1)."""
    hd, hkv = shape["head_dim"], shape["num_key_value_heads"]
    ctx, tables, nblk, pos, slots = decode_batch(batch, lo, hi, 256, seed)
    pool, k_cache, v_cache = paged_pool(nblk, 256, hkv, hd, seed + 2)
    g = torch.Generator().manual_seed(seed + 3)
    hidden = torch.randn(batch, shape["hidden_size"], generator=g).to(torch.bfloat16)
    residual = torch.randn(batch, shape["hidden_size"], generator=g).to(torch.bfloat16)
    ckpt = checkpoint(shape, seed, layers=1)
    layer = {k[len("model.layers.0."):]: v for k, v in ckpt.items() if k.startswith("model.layers.0.")}
    return dict(shape=shape, layer=layer, hidden=hidden, residual=residual, pool=pool, k_cache=k_cache,
                v_cache=v_cache, context_lens=ctx, block_tables=tables, positions=pos, slot_mapping=slots)


def host_workload():
    """Scripted request stream for the scheduler / metadata trace (block_size 4):
    shared prefixes, a prompt longer than the token budget (chunked prefill),
    a pool small enough to force preemption, and an eos stop."""
    base = [(7 * i + 3) % 89 + 1 for i in range(40)]
    prompts = [
        base[:30],                                # 0
        base[:16] + [5, 6, 7, 8, 9, 10, 11, 12],  # 1: 4 cached blocks once 0 is hashed
        [2, 4, 6, 8, 10, 12, 14],                 # 2
        [(3 * i) % 50 + 1 for i in range(70)],    # 3: longer than the 64-token budget
        [(3 * i) % 50 + 1 for i in range(70)],    # 4: identical to 3 (prefix hit on 17 blocks)
        base[:30],                                # 5: identical to 0
    ]
    params = [(12, False), (9, False), (20, False), (6, True), (7, True), (5, False)]
    arrivals = {0: [0, 1, 2], 3: [3], 6: [4, 5]}  # step -> request indices added before it
    config = dict(max_num_seqs=4, max_num_batched_tokens=64, eos=0, kvcache_block_size=4, num_kvcache_blocks=28)
    return prompts, params, arrivals, config


def host_token(req: int, step: int, length: int) -> int:
    """Deterministic 'sampled' token; request 2 emits eos (0) as its 4th completion token."""
    return (req * 31 + step * 7 + length) % 97 + 1


def _plain(v):
    if v is None or isinstance(v, (int, float, bool)):
        return v
    if hasattr(v, "tolist"):
        return v.tolist()
    return list(v)


def run_host_trace(make_seq, scheduler, meta_prefill, meta_decode, max_steps: int = 1000):
    """Drive ``scheduler`` through host_workload(); returns (per-step trace, completions).

    Each trace entry holds the scheduled request indices, the prefill flag,
    the metadata the model runner would upload (plain lists) and the tokens
    fed back to postprocess."""
    prompts, params, arrivals, _ = host_workload()
    seqs: dict[int, object] = {}
    trace = []
    last_arrival = max(arrivals)
    for step in range(max_steps):
        for r in arrivals.get(step, []):
            seqs[r] = make_seq(prompts[r], params[r])
            scheduler.add(seqs[r])
        if scheduler.is_finished():
            if step > last_arrival:
                break
            continue
        sched, is_prefill = scheduler.schedule()
        ids = {id(s): r for r, s in seqs.items()}
        reqs = [ids[id(s)] for s in sched]
        meta = meta_prefill(sched) if is_prefill else meta_decode(sched)
        tokens = [0 if (r == 2 and s.num_completion_tokens == 3) else host_token(r, step, len(s))
                  for r, s in zip(reqs, sched)]
        scheduler.postprocess(sched, tokens, is_prefill)
        trace.append({"step": step, "prefill": bool(is_prefill), "reqs": reqs, "tokens": tokens,
                      "meta": {k: _plain(v) for k, v in meta.items()}})
    return trace, {r: list(s.completion_token_ids) for r, s in seqs.items()}


def replay(gold: dict, run_step):
    """Teacher-forced replay of a greedy fixture (make_golden._greedy_run):
    yields (logits, step record) for the prefill and every decode step, and
    then appends the REFERENCE's tokens, so one near-tie cannot derail the
    rest. ``run_step(batch)`` returns the [B, vocab] logits of a step; the
    batch dict holds CPU tensors: is_prefill, input_ids, positions,
    slot_mapping (int32), and cu_seqlens (int32) for the prefill or
    context_lens / block_tables (int32) for a decode step. Block size 256,
    one block per sequence (gold["tables"])."""
    seqs = [list(p) for p in gold["prompts"]]
    tables = gold["tables"]
    i32 = torch.int32
    batch = dict(is_prefill=True,
                 input_ids=torch.tensor([t for s in seqs for t in s]),
                 positions=torch.tensor([i for s in seqs for i in range(len(s))]),
                 cu_seqlens=torch.tensor([0] + torch.tensor([len(s) for s in seqs]).cumsum(0).tolist(), dtype=i32),
                 slot_mapping=torch.tensor([tables[b][0] * 256 + i for b, s in enumerate(seqs) for i in range(len(s))],
                                           dtype=i32))
    for step in gold["steps"]:
        yield run_step(batch), step
        for b, t in enumerate(step["tokens"]):
            seqs[b].append(t)
        batch = dict(is_prefill=False,
                     input_ids=torch.tensor([s[-1] for s in seqs]),
                     positions=torch.tensor([len(s) - 1 for s in seqs]),
                     slot_mapping=torch.tensor([tables[b][0] * 256 + len(s) - 1 for b, s in enumerate(seqs)], dtype=i32),
                     context_lens=torch.tensor([len(s) for s in seqs], dtype=i32),
                     block_tables=torch.tensor(tables, dtype=i32))


def check_greedy_step(logits: torch.Tensor, step: dict, min_cos: float = 0.999, ulps: int = 2) -> int:
    """Logits cosine >= min_cos against the reference's row by row, and the
    argmax equal to the reference's token wherever the reference's two largest
    logits are more than `ulps` bf16 ulps (2^-7 each at |logit| < 2) apart.
    Returns the number of tokens compared."""
    logits = logits.float().cpu()
    if "logits" in step:
        cos = torch.nn.functional.cosine_similarity(logits, step["logits"].float(), dim=-1)
        assert cos.min().item() >= min_cos, cos
    checked = 0
    for b, (mine, ref, margin) in enumerate(zip(logits.argmax(-1).tolist(), step["tokens"], step["margins"])):
        if margin > ulps * 2.0 ** -7:
            assert mine == ref, (b, mine, ref, margin)
            checked += 1
    return checked


def replay_prefix_cache(gold: dict, run_step):
    """Teacher-forced replay of the prefix-cache fixture (make_golden.golden_prefix_cache):
    prefill A; prefill B's new tokens over the cached block 0 (cu_seqlens_k >
    cu_seqlens_q, block_tables given); then 4 decode steps of A and B. Yields
    (logits, step record); batches as in ``replay`` plus cu_seqlens_k and,
    for B's prefill, block_tables."""
    a, b_new, tables = gold["a_prompt"], gold["b_new"], gold["tables"]
    b = a[:256] + b_new
    i32 = torch.int32

    def slot(row, pos):
        return tables[row][pos // 256] * 256 + pos % 256

    n = len(a)
    batches = [dict(is_prefill=True, input_ids=torch.tensor(a), positions=torch.arange(n),
                    cu_seqlens=torch.tensor([0, n], dtype=i32), cu_seqlens_k=torch.tensor([0, n], dtype=i32),
                    slot_mapping=torch.tensor([slot(0, i) for i in range(n)], dtype=i32), block_tables=None),
               dict(is_prefill=True, input_ids=torch.tensor(b_new), positions=torch.arange(256, len(b)),
                    cu_seqlens=torch.tensor([0, len(b_new)], dtype=i32), cu_seqlens_k=torch.tensor([0, len(b)], dtype=i32),
                    slot_mapping=torch.tensor([slot(1, i) for i in range(256, len(b))], dtype=i32),
                    block_tables=torch.tensor([tables[1]], dtype=i32))]
    steps = gold["steps"]
    for batch, rec in zip(batches, steps[:2]):
        yield run_step(batch), rec
    seqs = [a + steps[0]["tokens"], b + steps[1]["tokens"]]
    for rec in steps[2:]:
        batch = dict(is_prefill=False, input_ids=torch.tensor([s[-1] for s in seqs]),
                     positions=torch.tensor([len(s) - 1 for s in seqs]),
                     slot_mapping=torch.tensor([slot(r, len(s) - 1) for r, s in enumerate(seqs)], dtype=i32),
                     context_lens=torch.tensor([len(s) for s in seqs], dtype=i32),
                     block_tables=torch.tensor(tables, dtype=i32))
        yield run_step(batch), rec
        for r, t in enumerate(rec["tokens"]):
            seqs[r].append(t)


def model_step(model, b: dict, device=None):
    """One forward of a product model (kavor_b200.models) over a replay batch:
    the batch's tensors moved to ``device``, the attention context set as
    ModelRunner.prepare_prefill / prepare_decode set it (cu_seqlens_k and
    block_tables for a prefill over cached blocks), logits returned."""
    from kavor_b200.utils.context import reset_context, set_context

    if device is not None:
        b = {k: v.to(device) if isinstance(v, torch.Tensor) else v for k, v in b.items()}
    if b["is_prefill"]:
        cu_q = b["cu_seqlens"]
        cu_k = b.get("cu_seqlens_k", cu_q)
        set_context(True, cu_q, cu_k, int((cu_q[1:] - cu_q[:-1]).max()), int((cu_k[1:] - cu_k[:-1]).max()),
                    b["slot_mapping"], None, b.get("block_tables"))
    else:
        set_context(False, slot_mapping=b["slot_mapping"], context_lens=b["context_lens"],
                    block_tables=b["block_tables"])
    try:
        with torch.inference_mode():
            return model.compute_logits(model(b["input_ids"], b["positions"]))
    finally:
        reset_context()
