"""The TP > 1 decode step split into two micro-batches (Config.decode_microbatches
= 2) on CPU ranks (gloo, world size 2), kernels swapped for the oracle.

Each rank builds its shard of the tiny Qwen3 model and replays the reference's
greedy fixture (tests/golden/make_golden.py) teacher-forced, with the fused
all-reduce + add+RMSNorm played by a gloo stand-in of TPAllReduce: the prefill
runs whole through the step's communicator, every decode step runs as two
halves through their own communicators. What is checked is the wiring above
the C ABI: the row ranges, each half's slices of the step metadata, the buffer
schedule of each communicator, the reassembly of the final rows. The logits
must pass the same greedy rule as the unsplit path and agree with it; the
streams and the attention turns need CUDA and are exercised by the GPU tests."""
import os
import socket

import torch

WORLD = 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class GlooComm:
    """TPAllReduce's interface over gloo: partial buffers in host memory, the
    sum in fp32 (the same on every rank), rounded to bf16, then the oracle's
    add+RMSNorm with the residual updated in place. Logs (buffer, tokens) of
    every call."""

    EMBED_BUFFER = 2

    def __init__(self, max_tokens: int, hidden: int):
        self.max_tokens = max_tokens
        self.buffers = [torch.zeros(max_tokens, hidden, dtype=torch.bfloat16) for _ in range(3)]
        self._next = 0
        self.calls = []

    def start_forward(self):
        self._next = 0

    def next_buffer(self, tokens):
        idx = self._next
        self._next ^= 1
        return idx, self.partial_buffer(idx, tokens)

    def partial_buffer(self, index, tokens):
        assert tokens <= self.max_tokens
        return self.buffers[index][:tokens]

    def reduce_norm(self, index, tokens, residual, weight, eps, mode=0):
        import torch.distributed as dist
        from oracle import ops

        self.calls.append((index, tokens))
        y = self.buffers[index][:tokens].float()
        dist.all_reduce(y)
        y = y.to(torch.bfloat16)
        if residual is None:
            return ops.rmsnorm(y, weight, eps), y.clone()
        out, r = ops.add_rmsnorm(y, residual, weight, eps)
        residual.copy_(r)
        return out, residual

    def close(self, group=None):
        pass


def _replay(model, cases, gold, cfg):
    for lyr in model.model.layers:  # fresh pages per replay
        pool = torch.zeros(8, 2, 256, cfg.num_key_value_heads // WORLD, 128, dtype=torch.bfloat16)
        lyr.self_attn.attn.k_cache = [pool[:, 0]]
        lyr.self_attn.attn.v_cache = [pool[:, 1]]
    steps = []
    for logits, rec in cases.replay(gold, lambda b: cases.model_step(model, b)):
        steps.append((None if logits is None else logits.float().clone(), rec))
    return steps


def _worker(rank, port, out):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests"), os.path.join(root, "tests", "golden")]
    import torch.distributed as dist

    dist.init_process_group("gloo", f"tcp://127.0.0.1:{port}", world_size=WORLD, rank=rank)
    try:
        import cases
        import test_model_wiring as wiring

        from kavor_b200 import _kernels as K
        from kavor_b200.layers import allreduce as AR
        from kavor_b200.models import AutoModelForCausalLM

        for name, fn in wiring.ORACLE_KERNELS:
            setattr(K, name, fn)
        torch.set_default_dtype(torch.bfloat16)
        cfg = cases.hf_config(cases.TINY)
        model = AutoModelForCausalLM.model_class(cfg)(cfg)
        AutoModelForCausalLM.load_weight(model, cfg, load_format="dummy", seed=5)  # the fixture's checkpoint
        from conftest import GOLDEN

        gold = torch.load(GOLDEN / "tiny_model_golden.pt", weights_only=False)
        H = cfg.hidden_size
        runs = {}
        for split in (False, True):
            main = GlooComm(512, H)
            halves = (GlooComm(8, H), GlooComm(8, H))
            AR.set_tp_allreduce(main)
            AR.set_decode_microbatches(AR.DecodeMicrobatches(halves, min_tokens=2) if split else None)
            try:
                steps = _replay(model, cases, gold, cfg)
            finally:
                AR.set_tp_allreduce(None)
                AR.set_decode_microbatches(None)
            runs[split] = (steps, main.calls, [h.calls for h in halves])
        out[rank] = runs
    finally:
        dist.destroy_process_group()


def test_microbatched_tp2_decode_replays_reference_greedy():
    import sys

    import torch.multiprocessing as mp

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import cases

    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _port()
        # CPU (gloo) ranks holding no device memory: daemonic, and ended if they hang
        ps = [ctx.Process(target=_worker, args=(r, port, out), daemon=True) for r in range(WORLD)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(timeout=600)
        for p in ps:
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
        assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
        runs = {r: out[r] for r in range(WORLD)}
    layers = cases.TINY["num_hidden_layers"]
    whole, split = runs[0][False], runs[0][True]
    n_steps = len(whole[0])
    # prefill through the step's communicator both times; decode steps whole,
    # or as halves of 2 and 1 rows, each half 2L+1 calls per step
    assert len(whole[1]) == n_steps * (2 * layers + 1)
    assert len(split[1]) == 2 * layers + 1
    for h, rows in enumerate((2, 1)):
        calls = split[2][h]
        assert len(calls) == (n_steps - 1) * (2 * layers + 1)
        assert all(t == rows for _, t in calls)
        idx = [i for i, _ in calls]
        assert all(a != b for a, b in zip(idx, idx[1:]))  # consecutive calls never share a buffer
    assert runs[1][True][2] == split[2]  # both ranks made the same calls in the same order
    checked = 0
    for (lw, rec), (ls, _) in zip(whole[0], split[0]):
        checked += cases.check_greedy_step(ls, rec, min_cos=0.9999)
        cos = torch.nn.functional.cosine_similarity(lw, ls, dim=-1)
        assert cos.min().item() >= 0.99999, cos
    assert checked >= 13
