"""Generate the golden fixtures of tests/golden from the REFERENCE implementation.

Run once in a container that has the reference source tree (it is never
needed on the GPU box):

    TORCH_COMPILE_DISABLE=1 python tests/golden/make_golden.py --reference <kavor checkout>

What runs is the reference's own code on the CPU:
* RMSNorm.rms_forward / add_rms_forward through their eager branches
  (layernorm.py:246-251, :283-288; forced by lowering _MAX_FUSED_COLS);
* RotaryEmbedding's cos_sin_cache (rotary_embedding.py:96-102) and the eager
  apply_rotary_emb / apply_rotary_emb_interleaved (:56-79);
* SiluAndMul with torch.compile disabled (activation.py:8-11, eager); for the
  Qwen3-8B layer case, its compiled numerics instead (fp32, one rounding:
  what torch.compile's fused kernel computes on the GPU);
* Qwen3DecoderLayer (qwen3.py:123-162) and Qwen3ForCausalLM (:189-219) with
  the reference's TP layers and weight loaders on a 1-rank gloo group. Its
  three non-CPU kernels are replaced: the Triton RoPE by the eager function
  above, store_kvcache (Triton) and the two flash_attn calls by oracle.ops
  (flash-attn is a third-party GPU wheel; that boundary is pinned on the GPU
  instead, by running the wheel beside the kernels:
  tests/test_flash_attn_parity_gpu.py);
* Scheduler + BlockManager + ModelRunner.prepare_prefill/prepare_decode
  (scheduler.py, block_manager.py, model_runner.py:385-473) on a scripted
  request stream, with the CUDA uploads turned into CPU no-ops;
* MistralForCausalLM and Ernie4_5ForCausalLM (mistral.py, ernie4_5.py) on
  tiny configs, the same greedy run as the Qwen3 model;
* the Qwen3 model over a cached prefix: a second prompt that reuses the
  first prompt's full block prefills only its new tokens against the paged
  cache, then both decode.

Outputs: ops_golden.pt, layer_golden.pt, layer_8b_golden.pt, tiny_model_golden.pt, tiny_model_golden_32.pt,
mistral_tiny_golden.pt, ernie4_5_tiny_golden.pt, prefix_cache_golden.pt, host_trace.json.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

os.environ.setdefault("TORCH_COMPILE_DISABLE", "1")

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

import cases  # noqa: E402
from oracle import ops  # noqa: E402


def _ref_patch_kernels():
    """Swap the reference's GPU-only kernels for CPU equivalents (see module doc)."""
    from kavor.layers import layernorm, rotary_embedding
    from kavor.layers.attention import flash_attention_kvcache as fak

    layernorm._MAX_FUSED_COLS = 0  # every RMSNorm call takes its eager branch

    def rope_forward(self, positions, query, key):
        cs = self.cos_sin_cache[positions]
        cos, sin = cs.chunk(2, dim=-1)
        f = rotary_embedding.apply_rotary_emb_interleaved if self.interleaved else rotary_embedding.apply_rotary_emb
        return f(query, cos, sin), f(key, cos, sin)

    rotary_embedding.RotaryEmbedding.forward = rope_forward

    def with_kvcache(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, causal):
        return ops.paged_decode_attention(q[:, 0], k_cache, v_cache, block_table, cache_seqlens,
                                          softmax_scale).unsqueeze(1)

    def varlen(q, k, v, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, softmax_scale, causal,
               block_table=None):
        return ops.varlen_prefill_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, softmax_scale, block_table)

    fak.flash_attn_with_kvcache = with_kvcache
    fak.flash_attn_varlen_func = varlen
    fak.store_kvcache = lambda key, value, k_cache, v_cache, slot_mapping: ops.store_kvcache(
        key, value, k_cache, v_cache, slot_mapping)


def golden_ops() -> dict:
    from kavor.layers.activation import SiluAndMul
    from kavor.layers.layernorm import RMSNorm
    from kavor.layers.rotary_embedding import RotaryEmbedding, apply_rotary_emb, apply_rotary_emb_interleaved

    out = {}
    g = torch.Generator().manual_seed(11)
    for name, shape, view in (("rms_2d", (7, 1024), False), ("rms_4096", (5, 4096), False),
                              ("rms_qk", (6, 16, 128), True)):
        norm = RMSNorm(shape[-1], eps=1e-6)
        with torch.no_grad():
            norm.weight.copy_((torch.randn(shape[-1], generator=g) * 0.1 + 1).to(torch.bfloat16))
        if view:
            buf = torch.randn(shape[0], shape[1] * 3, shape[2], generator=g).to(torch.bfloat16)
            x = buf[:, :shape[1], :]
        else:
            x = torch.randn(shape, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            out[name] = dict(x=x.contiguous(), w=norm.weight.detach().clone(), y=norm(x))
    norm = RMSNorm(4096, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_((torch.randn(4096, generator=g) * 0.1 + 1).to(torch.bfloat16))
        x = torch.randn(9, 4096, generator=g).to(torch.bfloat16)
        r = torch.randn(9, 4096, generator=g).to(torch.bfloat16)
        y, r2 = norm(x.clone(), r.clone())
    out["add_rms"] = dict(x=x, r=r, w=norm.weight.detach().clone(), y=y, r_out=r2)

    rope = RotaryEmbedding(128, 128, 4096, 1000000.0)
    rows = torch.arange(0, 4096, 61)
    out["rope_cache"] = dict(max_position=4096, rows=rows, values=rope.cos_sin_cache[rows].clone())
    T, Hq, Hkv = 12, 8, 2
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 4096, (T,), generator=g)
    cs = rope.cos_sin_cache[pos]
    cos, sin = cs.chunk(2, dim=-1)
    q = qkv[:, :Hq * 128].view(T, Hq, 128)
    k = qkv[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    out["rope"] = dict(qkv=qkv, pos=pos, q=apply_rotary_emb(q.clone(), cos, sin), k=apply_rotary_emb(k.clone(), cos, sin),
                       q_il=apply_rotary_emb_interleaved(q.clone(), cos, sin),
                       k_il=apply_rotary_emb_interleaved(k.clone(), cos, sin))
    x = torch.randn(10, 2 * 3072, generator=g).to(torch.bfloat16)
    out["silu"] = dict(x=x, y=SiluAndMul()(x))
    return out


def _ref_layer(shape_cfg):
    from kavor.models.qwen3 import Qwen3DecoderLayer

    torch.set_default_dtype(torch.bfloat16)
    try:
        layer = Qwen3DecoderLayer(shape_cfg)
    finally:
        torch.set_default_dtype(torch.float32)
    return layer


def _load_layer(layer, tensors: dict):
    packed = {"q_proj": ("qkv_proj", "q"), "k_proj": ("qkv_proj", "k"), "v_proj": ("qkv_proj", "v"),
              "gate_proj": ("gate_up_proj", 0), "up_proj": ("gate_up_proj", 1)}
    for name, t in tensors.items():
        for k, (v, sid) in packed.items():
            if k in name:
                p = layer.get_parameter(name.replace(k, v))
                p.weight_loader(p, t, sid)
                break
        else:
            p = layer.get_parameter(name)
            loader = getattr(p, "weight_loader", None)
            p.data.copy_(t) if loader is None else loader(p, t)


def _compiled_silu_and_mul(self, x):
    """activation.py:8-11 as the reference runs it on the GPU: torch.compile
    fuses silu(x) * y into one kernel that computes in fp32 and rounds once.
    Its eager form (what runs on the CPU with compilation disabled) rounds
    silu(x) to bf16 first; over the 12288 intermediate features of a Qwen3-8B
    MLP those extra roundings move the down projection's outputs by more than
    the per-layer bound, so the 8B layer case uses the compiled numerics."""
    g, u = x.float().chunk(2, -1)
    return (torch.nn.functional.silu(g) * u).to(x.dtype)


def golden_layer(case_fn=cases.config1_layer_case, compiled_silu: bool = False) -> dict:
    from kavor.layers.activation import SiluAndMul

    case = case_fn(0)
    eager_forward = SiluAndMul.forward
    if compiled_silu:
        SiluAndMul.forward = _compiled_silu_and_mul
    try:
        return _run_layer_case(case)
    finally:
        SiluAndMul.forward = eager_forward


def _run_layer_case(case) -> dict:
    from kavor.utils.context import reset_context, set_context

    layer = _ref_layer(cases.hf_config(case["shape"]))
    _load_layer(layer, case["layer"])
    attn = layer.self_attn.attn
    res = {}
    for variant in ("first", "later"):
        pool = case["pool"].clone()
        attn.k_cache = [pool[:, 0]]
        attn.v_cache = [pool[:, 1]]
        set_context(False, slot_mapping=case["slot_mapping"], context_lens=case["context_lens"],
                    block_tables=case["block_tables"])
        with torch.no_grad():
            h, r = layer(case["positions"], case["hidden"].clone(),
                         None if variant == "first" else case["residual"].clone())
        reset_context()
        res[variant] = dict(hidden=h, residual=r)
    return res


def golden_tiny_model(decode_steps: int = 8, keep_logits: bool = True) -> dict:
    """Greedy generation of a 2-layer Qwen3 (reference model class, CPU) for 3
    prompts: one prefill step then `decode_steps` decode steps, block_size 256.
    Every step keeps its tokens and the gap between the two largest logits of
    each row (a near-tie there is where a bf16 rounding difference may pick
    the other token); the logits themselves only with keep_logits."""
    from kavor.models.qwen3 import Qwen3ForCausalLM

    shape = cases.TINY
    model = _ref_model(Qwen3ForCausalLM, cases.hf_config(shape), cases.checkpoint(shape, seed=5))
    return _greedy_run(model, shape["num_key_value_heads"], decode_steps, keep_logits)


def golden_family_model(family: str, decode_steps: int = 8) -> dict:
    """The same greedy run on the tiny member of another dense family
    (reference classes mistral.py:147-175 / ernie4_5.py:180-209)."""
    from kavor.models.ernie4_5 import Ernie4_5ForCausalLM
    from kavor.models.mistral import MistralForCausalLM

    cls = {"mistral": MistralForCausalLM, "ernie4_5": Ernie4_5ForCausalLM}[family]
    cfg = cases.family_config(family)
    model = _ref_model(cls, cfg, cases.family_checkpoint(family, seed=5))
    return _greedy_run(model, cfg.num_key_value_heads, decode_steps, True)


def _ref_model(cls, cfg, ckpt: dict):
    torch.set_default_dtype(torch.bfloat16)
    try:
        model = cls(cfg)
    finally:
        torch.set_default_dtype(torch.float32)
    packed = cls.packed_modules_mapping
    for name, t in ckpt.items():
        for k, (v, sid) in packed.items():
            if k in name:
                p = model.get_parameter(name.replace(k, v))
                p.weight_loader(p, t, sid)
                break
        else:
            p = model.get_parameter(name)
            loader = getattr(p, "weight_loader", None)
            p.data.copy_(t) if loader is None else loader(p, t)
    return model


def _greedy_run(model, hkv: int, decode_steps: int, keep_logits: bool) -> dict:
    from kavor.utils.context import reset_context, set_context

    nblk = 8
    pools = [torch.zeros(nblk, 2, 256, hkv, 128, dtype=torch.bfloat16) for _ in model.model.layers]
    for lyr, pool in zip(model.model.layers, pools):
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]
    prompts = [[(13 * i + 7 * j) % 4000 + 3 for j in range(n)] for i, n in enumerate((37, 5, 100))]
    tables = [[0], [3], [5]]
    seqs = [list(p) for p in prompts]
    steps = []
    with torch.no_grad():
        ids = torch.tensor([t for p in seqs for t in p])
        pos = torch.tensor([i for p in seqs for i in range(len(p))])
        cu = torch.tensor([0] + list(torch.tensor([len(p) for p in seqs]).cumsum(0)), dtype=torch.int32)
        slots = torch.tensor([tables[b][0] * 256 + i for b, p in enumerate(seqs) for i in range(len(p))],
                             dtype=torch.int32)
        set_context(True, cu, cu, max(map(len, seqs)), max(map(len, seqs)), slots, None, None)
        logits = model.compute_logits(model(ids, pos))
        reset_context()
        steps.append(_step_record(logits, keep_logits))
        for b, t in enumerate(steps[-1]["tokens"]):
            seqs[b].append(t)
        for _ in range(decode_steps):
            ids = torch.tensor([p[-1] for p in seqs])
            pos = torch.tensor([len(p) - 1 for p in seqs])
            ctx = torch.tensor([len(p) for p in seqs], dtype=torch.int32)
            slots = torch.tensor([tables[b][0] * 256 + len(p) - 1 for b, p in enumerate(seqs)], dtype=torch.int32)
            set_context(False, slot_mapping=slots, context_lens=ctx, block_tables=torch.tensor(tables, dtype=torch.int32))
            logits = model.compute_logits(model(ids, pos))
            reset_context()
            steps.append(_step_record(logits, keep_logits))
            for b, t in enumerate(steps[-1]["tokens"]):
                seqs[b].append(t)
    return dict(prompts=prompts, tables=tables, steps=steps)


def golden_prefix_cache() -> dict:
    """The 2-layer Qwen3 (reference model class, CPU) over a cached prefix:
    prompt A (300 tokens, blocks [0, 1]) is prefilled; prompt B = A's first 256
    tokens + 40 new ones reuses block 0 (block table [0, 2]) and prefills only
    its 40 new tokens against the paged cache (flash_attention_kvcache.py:74-79
    with block_table); then A and B decode 4 greedy steps together."""
    from kavor.models.qwen3 import Qwen3ForCausalLM
    from kavor.utils.context import reset_context, set_context

    shape = cases.TINY
    model = _ref_model(Qwen3ForCausalLM, cases.hf_config(shape), cases.checkpoint(shape, seed=5))
    pool = torch.zeros(8, 2, 256, shape["num_key_value_heads"], 128, dtype=torch.bfloat16)
    pools = [pool.clone() for _ in model.model.layers]
    for lyr, pl in zip(model.model.layers, pools):
        lyr.self_attn.attn.k_cache = [pl[:, 0]]
        lyr.self_attn.attn.v_cache = [pl[:, 1]]
    a_prompt, b_new = cases.prefix_cache_prompts()
    b_prompt = a_prompt[:256] + b_new
    tables = [[0, 1], [0, 2]]
    i32 = torch.int32
    steps = []
    with torch.no_grad():
        # prefill A
        n = len(a_prompt)
        set_context(True, torch.tensor([0, n], dtype=i32), torch.tensor([0, n], dtype=i32), n, n,
                    torch.tensor([tables[0][i // 256] * 256 + i % 256 for i in range(n)], dtype=i32), None, None)
        logits = model.compute_logits(model(torch.tensor(a_prompt), torch.arange(n)))
        reset_context()
        steps.append(_step_record(logits, True))
        # prefill B's new tokens over the cached prefix (block 0)
        nq, nk = len(b_new), len(b_prompt)
        set_context(True, torch.tensor([0, nq], dtype=i32), torch.tensor([0, nk], dtype=i32), nq, nk,
                    torch.tensor([tables[1][i // 256] * 256 + i % 256 for i in range(256, nk)], dtype=i32), None,
                    torch.tensor([tables[1]], dtype=i32))
        logits = model.compute_logits(model(torch.tensor(b_new), torch.arange(256, nk)))
        reset_context()
        steps.append(_step_record(logits, True))
        seqs = [a_prompt + steps[0]["tokens"], b_prompt + steps[1]["tokens"]]
        for _ in range(4):
            ids = torch.tensor([p[-1] for p in seqs])
            pos = torch.tensor([len(p) - 1 for p in seqs])
            ctx = torch.tensor([len(p) for p in seqs], dtype=i32)
            slots = torch.tensor([tables[b][(len(p) - 1) // 256] * 256 + (len(p) - 1) % 256 for b, p in enumerate(seqs)],
                                 dtype=i32)
            set_context(False, slot_mapping=slots, context_lens=ctx, block_tables=torch.tensor(tables, dtype=i32))
            logits = model.compute_logits(model(ids, pos))
            reset_context()
            steps.append(_step_record(logits, True))
            for b, t in enumerate(steps[-1]["tokens"]):
                seqs[b].append(t)
    return dict(a_prompt=a_prompt, b_new=b_new, tables=tables, steps=steps)


def _step_record(logits: torch.Tensor, keep_logits: bool) -> dict:
    top2 = logits.float().topk(2, dim=-1).values
    rec = dict(tokens=logits.float().argmax(-1).tolist(), margins=(top2[:, 0] - top2[:, 1]).tolist())
    if keep_logits:
        rec["logits"] = logits.clone()
    return rec


def golden_host_trace() -> dict:
    from kavor.engine import model_runner as mr
    from kavor.engine.multimodal import PromptInputs
    from kavor.engine.scheduler import Scheduler
    from kavor.engine.sequence import Sequence
    from kavor.sampling_params import SamplingParams

    class _TorchNoUpload:
        """model_runner's torch handle with pinned/CUDA uploads made CPU no-ops."""

        def __getattr__(self, name):
            return getattr(torch, name)

        @staticmethod
        def tensor(data, dtype=None, pin_memory=False, **kw):
            return torch.tensor(data, dtype=dtype)

    captured = {}

    def fake_set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                         slot_mapping=None, context_lens=None, block_tables=None, *rest, **kw):
        captured.clear()
        captured.update(cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k, max_seqlen_q=max_seqlen_q,
                        max_seqlen_k=max_seqlen_k, slot_mapping=slot_mapping, context_lens=context_lens,
                        block_tables=block_tables)

    mr.torch = _TorchNoUpload()
    mr.set_context = fake_set_context
    orig_cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self
    fake_cache = SimpleNamespace(copy_blocks=lambda s, d: None, prepare_linear_slot_ids=lambda seqs: None,
                                 prepare_linear_cache_slot_ids=lambda seqs: None,
                                 check_linear_states=lambda seqs: None)
    prompts, params, arrivals, cfg = cases.host_workload()
    fake_runner = SimpleNamespace(block_size=cfg["kvcache_block_size"], cache=fake_cache)
    fake_runner.prepare_block_tables = lambda seqs: mr.ModelRunner.prepare_block_tables(fake_runner, seqs)
    Sequence.block_size = cfg["kvcache_block_size"]
    sched = Scheduler(SimpleNamespace(**cfg, has_linear_attention=False, num_linear_state_groups=0))

    def make_seq(prompt, p):
        return Sequence(PromptInputs(token_ids=list(prompt), prompt=""),
                        SamplingParams(temperature=1.0, max_tokens=p[0], ignore_eos=p[1]))

    def meta_prefill(seqs):
        ids, pos = mr.ModelRunner.prepare_prefill(fake_runner, seqs)
        return dict(input_ids=ids, positions=pos, **{k: captured[k] for k in (
            "cu_seqlens_q", "cu_seqlens_k", "max_seqlen_q", "max_seqlen_k", "slot_mapping", "block_tables")})

    def meta_decode(seqs):
        ids, pos = mr.ModelRunner.prepare_decode(fake_runner, seqs)
        return dict(input_ids=ids, positions=pos, slot_mapping=captured["slot_mapping"],
                    context_lens=captured["context_lens"], block_tables=captured["block_tables"])

    try:
        trace, final = cases.run_host_trace(make_seq, sched, meta_prefill, meta_decode)
    finally:
        torch.Tensor.cuda = orig_cuda
    bm = sched.block_manager
    return dict(trace=trace, completions={str(k): v for k, v in final.items()},
                prefix_cache_hit_tokens=bm.prefix_cache_hit_tokens,
                prefix_cache_prompt_tokens=bm.prefix_cache_prompt_tokens)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, help="root of the reference (Kavor) source tree")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29533", world_size=1, rank=0)
    _ref_patch_kernels()
    out = Path(args.out)
    torch.save(golden_ops(), out / "ops_golden.pt")
    torch.save(golden_layer(), out / "layer_golden.pt")
    torch.save(golden_layer(cases.config3_layer_case, compiled_silu=True), out / "layer_8b_golden.pt")
    torch.save(golden_tiny_model(), out / "tiny_model_golden.pt")
    torch.save(golden_tiny_model(decode_steps=31, keep_logits=False), out / "tiny_model_golden_32.pt")
    for family in cases.FAMILIES:
        torch.save(golden_family_model(family), out / f"{family}_tiny_golden.pt")
    torch.save(golden_prefix_cache(), out / "prefix_cache_golden.pt")
    (out / "host_trace.json").write_text(json.dumps(golden_host_trace()))
    dist.destroy_process_group()
    for f in sorted(out.glob("*golden*")) + [out / "host_trace.json"]:
        print(f.name, f.stat().st_size)
    return 0


if __name__ == "__main__":
    sys.exit(main())
