"""Host model of the decode micro-batch schedule (Config.decode_microbatches = 2).

The real ``Qwen3Model._forward_microbatched`` runs on the CPU (oracle kernels)
with torch's CUDA stream and event calls replaced by a recorder, so that what
is checked is the dependency graph the code actually issues: every kernel
launch, all-reduce call, stream fork / join and attention turn, per stream.

1. Ordering: each half's work stays in issue order on its own stream, the two
   halves' decode attention kernels alternate (A0, B0, A1, B1, ...: each
   depends on the previous one, which also keeps the shared split-KV scratch
   in use by one kernel at a time), and the step's end depends on both halves.
2. Deadlock freedom: that graph is executed on two simulated ranks, each a GPU
   of 148 SMs with two block slots per SM, under random block placement. An
   all-reduce block finishes only once the same block of the same call is
   resident on every rank (the kernel's spin on its peers); other blocks
   finish after a random delay. With the communicators' grid cap
   (DecodeMicrobatches.MAX_BLOCKS) every schedule completes; with grids as
   large as the GPU, the model finds the deadlock that the cap exists to
   exclude (a reduced two-stream graph, so that the model is shown to detect
   it)."""
import contextlib
import random

import pytest
import torch

import cases

SMS, SLOTS = 148, 2


class Recorder:
    """Kernel launches and stream dependencies as the code issues them."""

    def __init__(self):
        self.ops = []       # dicts: kind, stream, deps, info
        self.last = {}      # stream name -> index of its last op
        self.waits = {}     # stream name -> ops its next op must wait for
        self.cur = ["main"]

    def op(self, kind, **info):
        s = self.cur[-1]
        deps = set(self.waits.pop(s, set()))
        if s in self.last:
            deps.add(self.last[s])
        self.ops.append(dict(kind=kind, stream=s, deps=deps, **info))
        self.last[s] = len(self.ops) - 1
        return len(self.ops) - 1


class FakeStream:
    def __init__(self, rec, name):
        self.rec, self.name = rec, name

    def wait_stream(self, other):
        if other.name in self.rec.last:
            self.rec.waits.setdefault(self.name, set()).add(self.rec.last[other.name])

    def wait_event(self, ev):
        if ev.op is not None:
            self.rec.waits.setdefault(self.name, set()).add(ev.op)


class FakeEvent:
    rec = None

    def __init__(self, *a, **k):
        self.op = None

    def record(self, stream=None):
        self.op = self.rec.last.get(stream.name if stream is not None else self.rec.cur[-1])


class RecComm:
    """TPAllReduce's interface on one process (the sum of one partial); each
    call is recorded as an all-reduce launch of this communicator."""

    EMBED_BUFFER = 2

    def __init__(self, rec, cid, max_tokens, hidden):
        self.rec, self.cid, self.max_tokens = rec, cid, max_tokens
        self.buffers = [torch.zeros(max_tokens, hidden, dtype=torch.bfloat16) for _ in range(3)]
        self._next = 0
        self.calls = 0

    def start_forward(self):
        self._next = 0

    def next_buffer(self, tokens):
        idx = self._next
        self._next ^= 1
        return idx, self.buffers[idx][:tokens]

    def partial_buffer(self, index, tokens):
        return self.buffers[index][:tokens]

    def reduce_norm(self, index, tokens, residual, weight, eps, mode=0):
        from oracle import ops

        self.rec.op("ar", comm=self.cid, call=self.calls, rows=tokens)
        self.calls += 1
        y = self.buffers[index][:tokens].clone()
        if residual is None:
            return ops.rmsnorm(y, weight, eps), y
        out, r = ops.add_rmsnorm(y, residual, weight, eps)
        residual.copy_(r)
        return out, residual


@pytest.fixture(scope="module")
def graph():
    """The op graph of one micro-batched decode step of a 4-layer tiny Qwen3
    (6 sequences: halves of 3)."""
    import test_model_wiring as wiring

    from kavor_b200 import _kernels as K
    from kavor_b200.layers import allreduce as AR
    from kavor_b200.layers import linear as L
    from kavor_b200.models import AutoModelForCausalLM
    from kavor_b200.utils.context import reset_context, set_context

    rec = Recorder()
    mp = pytest.MonkeyPatch()
    try:
        for name, fn in wiring.ORACLE_KERNELS:
            kind = "attn" if name == "paged_decode_attention" else "work"
            mp.setattr(K, name, lambda *a, _f=fn, _k=kind, _n=name, **k: (rec.op(_k, name=_n), _f(*a, **k))[1])
        gemm = L.linear
        mp.setattr(L, "linear", lambda *a, **k: (rec.op("work", name="gemm"), gemm(*a, **k))[1])
        side = FakeStream(rec, "side")
        main = FakeStream(rec, "main")
        FakeEvent.rec = rec

        @contextlib.contextmanager
        def on(stream):
            rec.cur.append(stream.name)
            try:
                yield
            finally:
                rec.cur.pop()

        mp.setattr(torch.cuda, "current_stream", lambda *a, **k: FakeStream(rec, rec.cur[-1]))
        mp.setattr(torch.cuda, "stream", on)
        mp.setattr(torch.cuda, "Event", FakeEvent)

        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            cfg = cases.hf_config(cases.TINY, num_hidden_layers=4)
            model = AutoModelForCausalLM.model_class(cfg)(cfg)
        finally:
            torch.set_default_dtype(prev)
        AutoModelForCausalLM.load_weight(model, cfg, load_format="dummy", seed=1)
        ctx, tables, nblk, pos, slots = cases.decode_batch(6, 50, 600, 256, seed=3)
        for lyr in model.model.layers:
            pool = torch.zeros(nblk, 2, 256, cfg.num_key_value_heads, 128, dtype=torch.bfloat16)
            lyr.self_attn.attn.k_cache = [pool[:, 0]]
            lyr.self_attn.attn.v_cache = [pool[:, 1]]
        comms = (RecComm(rec, 0, 8, cfg.hidden_size), RecComm(rec, 1, 8, cfg.hidden_size))
        mb = AR.DecodeMicrobatches(comms, min_tokens=2, side_stream=side)
        set_context(False, slot_mapping=slots, context_lens=ctx, block_tables=tables)
        try:
            with torch.inference_mode():
                out = model.model._forward_microbatched(mb, torch.arange(6) + 5, pos)
        finally:
            reset_context()
        with on(main):
            end = rec.op("end")  # the step's end on the launching stream (what the sampler waits for)
    finally:
        mp.undo()
    assert out.shape == (6, cfg.hidden_size) and torch.isfinite(out.float()).all()
    return rec.ops, end, cfg.num_hidden_layers


def _ancestors(ops, i):
    seen, todo = set(), list(ops[i]["deps"])
    while todo:
        j = todo.pop()
        if j not in seen:
            seen.add(j)
            todo.extend(ops[j]["deps"])
    return seen


def test_halves_run_on_their_streams_and_attention_kernels_alternate(graph):
    ops, end, layers = graph
    attn = [i for i, o in enumerate(ops) if o["kind"] == "attn"]
    assert [ops[i]["stream"] for i in attn] == ["main", "side"] * layers
    for a, b in zip(attn, attn[1:]):
        assert a in _ancestors(ops, b)  # every attention waits for the previous one
    for cid, stream in ((0, "main"), (1, "side")):
        calls = [o for o in ops if o["kind"] == "ar" and o["comm"] == cid]
        assert len(calls) == 2 * layers + 1 and all(o["stream"] == stream for o in calls)
        assert all(o["rows"] == 3 for o in calls)
    anc = _ancestors(ops, end)
    assert all(i in anc for i, o in enumerate(ops) if o["kind"] != "end")  # the join covers both halves


def _simulate(ops, ar_blocks, seed, ranks=2, work_blocks=(148, 1), attn_blocks=(64, 2), skew=False,
              max_ticks=20000):
    """Run the op graph on `ranks` simulated GPUs; True when every op completes,
    False on a deadlock (nothing can be placed and nothing can finish). Blocks
    of a kernel are dispatched in index order to the least-loaded SM with room
    (breadth first, as the hardware spreads a grid), kernels in random order.
    ``skew``: rank 0 runs the first half's kernels fast and the second half's
    slowly, rank 1 the reverse, so the halves drift apart in opposite
    directions on the two ranks."""
    rng = random.Random(seed)
    n = len(ops)
    size = []
    for o in ops:
        if o["kind"] == "ar":
            size.append((min(o["rows"], ar_blocks), 1))
        elif o["kind"] == "attn":
            size.append(attn_blocks)
        elif o["kind"] == "end":
            size.append((1, 1))
        else:
            size.append(work_blocks)
    free = [[SLOTS] * SMS for _ in range(ranks)]
    placed = [[0] * n for _ in range(ranks)]       # blocks dispatched so far (in index order)
    running = [dict() for _ in range(ranks)]        # (op, block) -> SM
    finished = [[0] * n for _ in range(ranks)]
    done = [[False] * n for _ in range(ranks)]
    for _ in range(max_ticks):
        progress = False
        for r in range(ranks):
            ready = [i for i in range(n) if not done[r][i] and placed[r][i] < size[i][0]
                     and all(done[r][d] for d in ops[i]["deps"])]
            rng.shuffle(ready)
            for i in ready:
                while placed[r][i] < size[i][0]:
                    need = size[i][1]
                    best = max(free[r])
                    if best < need:
                        break
                    s = rng.choice([k for k in range(SMS) if free[r][k] == best])
                    free[r][s] -= need
                    running[r][(i, placed[r][i])] = s
                    placed[r][i] += 1
                    progress = True
        for r in range(ranks):
            for (i, b), s in list(running[r].items()):
                if ops[i]["kind"] == "ar":
                    # spins until block b of this call has been dispatched on every rank
                    if not all(placed[q][i] > b for q in range(ranks)):
                        continue
                else:
                    fast = (ops[i]["stream"] == "main") == (r == 0)
                    if rng.random() < (0.3 if not skew else 0.1 if fast else 0.9):
                        continue
                del running[r][(i, b)]
                free[r][s] += size[i][1]
                finished[r][i] += 1
                progress = True
                if finished[r][i] == size[i][0]:
                    done[r][i] = True
        if all(all(d) for d in done):
            return True
        waiting = any(ops[i]["kind"] != "ar" for r in range(ranks) for i, _ in running[r])
        if not progress and not waiting:  # only spinning all-reduce blocks are left, and nothing fits
            return False
    raise AssertionError("simulation did not settle")


def _without_turns(ops):
    """The same graph without the attention turns (cross-stream waits of the
    attention kernels): only stream order, fork and join remain."""
    return [dict(o, deps={d for d in o["deps"] if ops[d]["stream"] == o["stream"]}) if o["kind"] == "attn" else o
            for o in ops]


@pytest.mark.parametrize("turns", [True, False])
def test_capped_grids_never_deadlock(graph, turns):
    """Halves of 128 rows (B = 256) with grids capped at MAX_BLOCKS: two
    spinning calls hold at most 128 of the 296 slots, so kernels that need a
    whole SM still find one; every schedule completes, with or without the
    attention turns."""
    from kavor_b200.layers.allreduce import DecodeMicrobatches

    ops, _, _ = graph
    ops = ops if turns else _without_turns(ops)
    rows = [dict(o, rows=128) if o["kind"] == "ar" else o for o in ops]
    for seed in range(16):
        assert _simulate(rows, DecodeMicrobatches.MAX_BLOCKS, seed, skew=seed % 2 == 1), seed


def _two_stream_pattern(rows):
    """The pattern the cap excludes, reduced to one layer half per stream:
    work, an attention kernel that needs a whole SM, then an all-reduce call,
    on each of the two streams."""
    ops = []
    for stream in ("main", "side"):
        base = len(ops)
        ops += [dict(kind="work", stream=stream, deps=set()),
                dict(kind="attn", stream=stream, deps={base}),
                dict(kind="ar", stream=stream, deps={base + 1}, rows=rows)]
    ops.append(dict(kind="end", stream="main", deps={2, 5}))
    return ops


def test_model_finds_the_deadlock_that_the_cap_excludes():
    """Sanity check of the model: with grids as large as the GPU's 296 block
    slots, rank 0 spinning in the first half's call and rank 1 in the second
    half's leave neither rank an SM for the attention kernel that precedes the
    other call, and the model reports the deadlock; capped at MAX_BLOCKS, the
    same schedules complete."""
    from kavor_b200.layers.allreduce import DecodeMicrobatches

    ops = _two_stream_pattern(SMS * SLOTS)
    assert not all(_simulate(ops, SMS * SLOTS, seed, skew=True) for seed in range(16))
    assert all(_simulate(ops, DecodeMicrobatches.MAX_BLOCKS, seed, skew=True) for seed in range(16))
