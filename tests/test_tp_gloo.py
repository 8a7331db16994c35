"""Multi-rank host logic on CPU ranks (gloo, world size 2): tensor-parallel
weight sharding, the cache-size agreement, the TP control-plane mailbox and
the decode-step all-reduce buffer schedule. No GPU is used."""
import os
import socket
from types import SimpleNamespace

import pytest
import torch

WORLD = 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_cfg(family="qwen3"):
    import cases

    return cases.hf_config(cases.TINY) if family == "qwen3" else cases.family_config(family)


def _shard_worker(rank, port, out, family):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests", "golden")]
    import torch.distributed as dist

    dist.init_process_group("gloo", f"tcp://127.0.0.1:{port}", world_size=WORLD, rank=rank)
    try:
        from kavor_b200.engine.cache_pool import CachePool
        from kavor_b200.models import AutoModelForCausalLM

        torch.set_default_dtype(torch.bfloat16)
        cfg = _tiny_cfg(family)
        model = AutoModelForCausalLM.model_class(cfg)(cfg)
        AutoModelForCausalLM.load_weight(model, cfg, load_format="dummy", seed=4)
        pool = CachePool(model, SimpleNamespace(), WORLD)
        agreed = pool._all_reduce_min(100 + 7 * rank)
        out[rank] = ({k: v.clone() for k, v in model.state_dict().items()}, agreed)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("family", ["qwen3", "ernie4_5"])  # ernie4_5: q/k/v biases shard with their rows
def test_tp2_shards_reassemble_the_tp1_weights(family):
    import torch.multiprocessing as mp

    from kavor_b200.models import AutoModelForCausalLM

    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _port()
        ps = [ctx.Process(target=_shard_worker, args=(r, port, out, family)) for r in range(WORLD)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(timeout=300)
        assert all(p.exitcode == 0 for p in ps)
        shards = [out[r][0] for r in range(WORLD)]
        assert out[0][1] == out[1][1] == 100  # MIN over ranks
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        cfg = _tiny_cfg(family)
        full = AutoModelForCausalLM.model_class(cfg)(cfg)
        AutoModelForCausalLM.load_weight(full, cfg, load_format="dummy", seed=4)
    finally:
        torch.set_default_dtype(prev)
    ref = full.state_dict()
    hq, hkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, 128
    for name, w in ref.items():
        parts = [s[name] for s in shards]
        if "qkv_proj" in name:  # per rank [q | k | v]
            qs, ks = hq // WORLD * hd, hkv // WORLD * hd
            q = torch.cat([p[:qs] for p in parts])
            k = torch.cat([p[qs:qs + ks] for p in parts])
            v = torch.cat([p[qs + ks:] for p in parts])
            assert torch.equal(torch.cat([q, k, v]), w), name
        elif "gate_up_proj" in name:  # per rank [gate | up]
            i = parts[0].shape[0] // 2
            assert torch.equal(torch.cat([p[:i] for p in parts] + [p[i:] for p in parts]), w), name
        elif "o_proj" in name or "down_proj" in name:
            assert torch.equal(torch.cat(parts, dim=1), w), name
        elif "embed_tokens" in name or "lm_head" in name:
            assert torch.equal(torch.cat(parts, dim=0), w), name
        else:  # replicated norms
            assert all(torch.equal(p, w) for p in parts), name


def _mailbox_worker(name, event, conn):
    from multiprocessing.shared_memory import SharedMemory

    from kavor_b200.engine.model_runner import ModelRunner

    shm = SharedMemory(name=name)
    calls = []
    runner = SimpleNamespace(shm=shm, event=event, world_size=WORLD, rank=1)
    while True:
        method, args = ModelRunner.read_shm(runner)
        calls.append((method, args))
        if method == "exit":
            break
    conn.send(calls)
    shm.close()


def test_mailbox_carries_calls_to_workers():
    """Rank 0 -> worker RPC (model_runner.py:85-112 semantics): pickled calls,
    one event per worker, decode sequences carry only their last token."""
    import multiprocessing as mp
    from multiprocessing.shared_memory import SharedMemory

    from kavor_b200.engine.model_runner import SHM_BYTES, ModelRunner
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    ctx = mp.get_context("spawn")
    name = f"kvb_test_{os.getpid()}"
    shm = SharedMemory(name=name, create=True, size=SHM_BYTES)
    try:
        ev = ctx.Event()
        recv, send = ctx.Pipe(duplex=False)
        p = ctx.Process(target=_mailbox_worker, args=(name, ev, send))
        p.start()
        runner = SimpleNamespace(shm=shm, event=[ev], world_size=WORLD, rank=0)
        seq = Sequence(list(range(1, 600)), SamplingParams(max_tokens=3))
        seq.block_table = [4, 9, 2]
        ModelRunner.write_shm(runner, "run", [seq], True)
        while ev.is_set():
            pass
        seq.is_prefill = False
        seq.append_token(77)
        ModelRunner.write_shm(runner, "run", [seq], False)
        while ev.is_set():
            pass
        ModelRunner.write_shm(runner, "exit")
        calls = recv.recv()
        p.join(timeout=60)
        assert p.exitcode == 0
        (m1, a1), (m2, a2), (m3, _) = calls
        assert (m1, m2, m3) == ("run", "run", "exit")
        assert a1[0][0].token_ids == list(range(1, 600)) and a1[1] is True
        assert a2[0][0].token_ids == [] and a2[0][0].last_token == 77 and a2[0][0].block_table == [4, 9, 2]
        with pytest.raises(RuntimeError, match="mailbox"):
            ModelRunner.write_shm(runner, "run", [b"x" * SHM_BYTES])
    finally:
        shm.close()
        shm.unlink()


def _slow_mailbox_worker(name, event, conn, delay):
    import time
    from multiprocessing.shared_memory import SharedMemory

    from kavor_b200.engine.model_runner import ModelRunner

    shm = SharedMemory(name=name)
    calls = []
    runner = SimpleNamespace(shm=shm, event=event, world_size=WORLD, rank=1)
    while True:
        time.sleep(delay)  # a worker still busy with its previous step
        method, args = ModelRunner.read_shm(runner)
        calls.append((method, args))
        if method == "exit":
            break
    conn.send(calls)
    shm.close()


def test_mailbox_writes_wait_for_a_slow_worker():
    """Calls that return before their step completes (run_async) can reach
    the mailbox again before a worker has read the last message: the write
    waits until every worker has taken it, so no message is overwritten."""
    import multiprocessing as mp
    from multiprocessing.shared_memory import SharedMemory

    from kavor_b200.engine.model_runner import SHM_BYTES, ModelRunner

    ctx = mp.get_context("spawn")
    name = f"kvb_slow_{os.getpid()}"
    shm = SharedMemory(name=name, create=True, size=SHM_BYTES)
    try:
        ev = ctx.Event()
        recv, send = ctx.Pipe(duplex=False)
        p = ctx.Process(target=_slow_mailbox_worker, args=(name, ev, send, 0.3))
        p.start()
        runner = SimpleNamespace(shm=shm, event=[ev], world_size=WORLD, rank=0)
        try:
            for i in range(4):  # back to back, no waiting on the caller's side
                ModelRunner.write_shm(runner, "run_async", [f"step{i}"], i > 0)
            ModelRunner.write_shm(runner, "exit")
            assert recv.poll(60), "the worker never saw its exit message"
            calls = recv.recv()
            p.join(timeout=60)
            assert p.exitcode == 0
        finally:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
        assert calls == [("run_async", [["step0"], False]), ("run_async", [["step1"], True]),
                         ("run_async", [["step2"], True]), ("run_async", [["step3"], True]), ("exit", [])]
    finally:
        shm.close()
        shm.unlink()


def test_model_steps_reach_workers_as_metadata_arrays():
    """ModelRunner.call("run" / "run_async", seqs, ...) on rank 0 builds the
    step's metadata once and sends the arrays: the worker receives the
    prefill_metadata / decode_metadata of the same sequences (and their
    temperatures) bit for bit, and rank 0 runs its own step from them."""
    import multiprocessing as mp
    from multiprocessing.shared_memory import SharedMemory

    import numpy as np

    from kavor_b200.engine.model_runner import SHM_BYTES, ModelRunner, decode_metadata, prefill_metadata
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    ctx = mp.get_context("spawn")
    name = f"kvb_meta_{os.getpid()}"
    shm = SharedMemory(name=name, create=True, size=SHM_BYTES)
    try:
        ev = ctx.Event()
        recv, send = ctx.Pipe(duplex=False)
        p = ctx.Process(target=_mailbox_worker, args=(name, ev, send))
        p.start()
        try:
            runner = ModelRunner.__new__(ModelRunner)
            runner.shm, runner.event, runner.world_size, runner.rank, runner.block_size = shm, [ev], WORLD, 0, 256
            local = []
            runner.run_step = lambda *a: local.append(("run_step", a)) or [0]
            runner.run_async_step = lambda *a: local.append(("run_async_step", a))
            seqs = [Sequence(list(range(1, 300 + 7 * i)), SamplingParams(temperature=0.5 + i, max_tokens=9))
                    for i in range(3)]
            for i, s in enumerate(seqs):
                s.block_table = [2 * i, 2 * i + 1]
                s.num_scheduled_tokens = s.num_tokens - 256 * (i == 1)  # sequence 1 has a cached first block
                s.num_cached_tokens = 256 * (i == 1)
            want_prefill = prefill_metadata(seqs, 256)
            runner.call("run", seqs, True)
            for s in seqs:
                s.num_cached_tokens, s.is_prefill = s.num_tokens, False
                s.append_token(40 + s.seq_id % 7)
            want_decode = decode_metadata(seqs, 256)
            runner.call("run", seqs, False)
            runner.call("run_async", seqs, [2, 0, 1])
            ModelRunner.write_shm(runner, "exit")
            assert recv.poll(60), "the worker never saw its exit message"
            calls = recv.recv()
            p.join(timeout=60)
            assert p.exitcode == 0
        finally:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
        temps = np.array([0.5, 1.5, 2.5], np.float32)
        expect = [("run_step", (want_prefill, temps, True)), ("run_step", (want_decode, temps, False)),
                  ("run_async_step", (want_decode, temps, [2, 0, 1]))]
        assert [m for m, _ in calls] == [m for m, _ in expect] + ["exit"]
        for (m, got), (_, (meta, t, last)), (lm, mine) in zip(calls, expect, local):
            assert lm == m
            for args in (tuple(got), mine):
                assert args[2] == last and np.array_equal(args[1], t)
                assert args[0].keys() == meta.keys()
                for k, v in meta.items():
                    assert (args[0][k] is None) if v is None else np.array_equal(args[0][k], v), (m, k)
    finally:
        shm.close()
        shm.unlink()


def test_allreduce_buffer_schedule_never_reuses_consecutively():
    """The decode step's 2L+1 fused all-reduces alternate data buffers so two
    consecutive reductions (also across steps) never share one."""
    from kavor_b200.layers.allreduce import TPAllReduce

    sched = SimpleNamespace(_next=0)
    seq = []
    for _ in range(3):  # three forwards
        TPAllReduce.start_forward(sched)
        seq.append(TPAllReduce.EMBED_BUFFER)
        for _ in range(36 * 2):
            sched_idx = sched._next
            sched._next ^= 1
            seq.append(sched_idx)
    assert all(a != b for a, b in zip(seq, seq[1:]))
