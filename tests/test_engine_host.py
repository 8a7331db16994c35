"""Host-side behaviour of Sequence, BlockManager and Scheduler, case by case —
the behaviours the reference's own suite checks for the full-attention path
(tests/test_sequence.py, test_block_manager.py, test_scheduler.py there), on
this package's classes, with 4-token blocks. (The golden host trace in
test_host_metadata.py checks the same classes end to end, bit-exact against a
trace produced by the reference.)"""
import pickle

import pytest

from kavor_b200.engine.block_manager import BlockManager
from kavor_b200.engine.scheduler import Scheduler
from kavor_b200.engine.sequence import SequenceStatus

BS = 4


# ------------------------------------------------------------------ Sequence
def test_sequence_block_arithmetic(make_seq):
    s = make_seq(range(1, 10))  # 9 tokens: blocks of 4, 4, 1
    assert s.num_blocks == 3 and s.last_block_num_tokens == 1
    assert s.block(0) == [1, 2, 3, 4] and s.block(2) == [9]
    with pytest.raises(IndexError):
        s.block(3)
    full = make_seq(range(8))
    assert full.num_blocks == 2 and full.last_block_num_tokens == 4


def test_append_token_advances_counters(make_seq):
    s = make_seq([5, 6, 7])
    s.append_token(42)
    assert len(s) == 4 and s.last_token == 42 and s.num_completion_tokens == 1
    assert s.completion_token_ids == [42] and s.prompt_token_ids == [5, 6, 7]


def test_pickle_sends_all_tokens_in_prefill_and_only_the_last_in_decode(make_seq):
    s = make_seq(range(10, 20))
    s.block_table = [3, 7, 1]
    p = pickle.loads(pickle.dumps(s))
    assert p.token_ids == list(range(10, 20)) and p.block_table == [3, 7, 1] and len(p) == 10
    s.is_prefill = False
    s.append_token(99)
    d = pickle.loads(pickle.dumps(s))
    assert d.token_ids == [] and d.last_token == 99 and len(d) == 11 and d.block_table == [3, 7, 1]


# ------------------------------------------------------------------ BlockManager
def _finish_prefill(bm, seq):
    """Allocate, run the whole prompt as one step and key its full blocks."""
    cached, _ = bm.can_allocate_prefill(seq)
    bm.allocate_prefill(seq, cached)
    seq.num_scheduled_tokens = len(seq) - seq.num_cached_tokens
    bm.hash_blocks(seq)
    seq.num_cached_tokens += seq.num_scheduled_tokens
    seq.num_scheduled_tokens = 0
    return cached


def test_allocate_then_free_restores_the_pool(make_seq):
    bm = BlockManager(8, BS)
    s = make_seq(range(10))
    bm.allocate_prefill(s, 0)
    assert s.block_table == [0, 1, 2] and len(bm.free_block_ids) == 5
    bm.deallocate(s)
    assert s.block_table == [] and len(bm.free_block_ids) == 8 and not bm.used_block_ids
    assert list(bm.free_block_ids)[-3:] == [2, 1, 0]  # freed last block first


def test_prefix_of_a_finished_sequence_is_reused(make_seq):
    bm = BlockManager(16, BS)
    a = make_seq(list(range(12)) + [100])  # 3 full blocks + 1 token
    _finish_prefill(bm, a)
    table_a = list(a.block_table)
    bm.deallocate(a)
    b = make_seq(list(range(12)) + [200, 201])
    cached, _ = bm.can_allocate_prefill(b)
    bm.allocate_prefill(b, cached)
    assert cached == 3 and b.block_table[:3] == table_a[:3] and b.num_cached_tokens == 12


def test_prefix_hits_stop_at_the_first_divergent_block(make_seq):
    bm = BlockManager(16, BS)
    _finish_prefill(bm, make_seq(list(range(12)) + [1]))
    b = make_seq([0, 1, 2, 3, 4, 5, 99, 7, 8, 9, 10, 11, 1])
    assert bm.can_allocate_prefill(b)[0] == 1


def test_the_last_block_of_a_prompt_is_never_served_from_the_cache(make_seq):
    bm = BlockManager(16, BS)
    _finish_prefill(bm, make_seq(range(8)))  # exactly two full blocks, both keyed
    same = make_seq(range(8))
    assert bm.can_allocate_prefill(same)[0] == 1  # its own last block is recomputed
    longer = make_seq(list(range(8)) + [50])
    assert bm.can_allocate_prefill(longer)[0] == 2  # but a longer prompt reuses both


def test_a_key_whose_block_holds_other_tokens_is_not_reused(make_seq):
    bm = BlockManager(16, BS)
    a = make_seq(list(range(8)) + [1])
    _finish_prefill(bm, a)
    bm.blocks[a.block_table[0]].token_ids = [9, 9, 9, 9]  # stale content behind a matching key
    assert bm.can_allocate_prefill(make_seq(list(range(8)) + [2]))[0] == 0


def test_sharing_a_running_prefix_counts_references(make_seq):
    bm = BlockManager(16, BS)
    a = make_seq(list(range(8)) + [1])
    _finish_prefill(bm, a)
    b = make_seq(list(range(8)) + [2])
    assert _finish_prefill(bm, b) == 2
    shared = a.block_table[:2]
    assert b.block_table[:2] == shared and all(bm.blocks[i].ref_count == 2 for i in shared)
    bm.deallocate(a)
    assert all(bm.blocks[i].ref_count == 1 and i in bm.used_block_ids for i in shared)


def test_allocation_reports_a_pool_too_small(make_seq):
    bm = BlockManager(2, BS)
    assert bm.can_allocate_prefill(make_seq(range(9)))[0] == -1
    assert bm.can_allocate_prefill(make_seq(range(8)))[0] == 0


def test_reallocating_a_freed_keyed_block_drops_its_key(make_seq):
    bm = BlockManager(2, BS)
    a = make_seq(list(range(4)) + [1])
    _finish_prefill(bm, a)
    key = bm.blocks[a.block_table[0]].hash
    assert bm.hash_to_block_id[key] == a.block_table[0]
    bm.deallocate(a)
    bm.allocate_block()
    bm.allocate_block()  # both blocks handed out again: the old key must be gone
    assert key not in bm.hash_to_block_id


def test_decode_takes_a_new_block_only_after_a_boundary(make_seq):
    bm = BlockManager(8, BS)
    s = make_seq(range(4))
    bm.allocate_prefill(s, 0)
    grown = []
    for t in range(9):
        s.append_token(t)
        before = len(s.block_table)
        bm.may_append_block(s)
        grown.append(len(s.block_table) - before)
    assert grown == [1, 0, 0, 0, 1, 0, 0, 0, 1]  # lengths 5, 9, 13 start a block


# ------------------------------------------------------------------ Scheduler
def _step(sched, token=7):
    seqs, is_prefill = sched.schedule()
    sched.postprocess(seqs, [token] * len(seqs), is_prefill)
    return seqs, is_prefill


def test_one_sequence_prefills_then_decodes(make_seq, make_config):
    sched = Scheduler(make_config())
    s = make_seq(range(1, 6), max_tokens=3, ignore_eos=True)
    sched.add(s)
    assert s.status == SequenceStatus.WAITING
    seqs, pre = _step(sched)
    assert pre and seqs == [s] and s.status == SequenceStatus.RUNNING and len(s) == 6
    seqs, pre = _step(sched)
    assert not pre and len(s) == 7
    _step(sched)
    assert s.status == SequenceStatus.FINISHED and sched.is_finished() and s.block_table == []


def test_a_long_prompt_is_chunked_by_the_token_budget(make_seq, make_config):
    sched = Scheduler(make_config(max_num_batched_tokens=8))
    s = make_seq(range(1, 21), ignore_eos=True)
    sched.add(s)
    sizes = []
    while True:
        seqs, pre = sched.schedule()
        if not pre:
            break
        sizes.append(s.num_scheduled_tokens)
        sched.postprocess(seqs, [7], pre)
    assert sizes == [8, 8, 4] and len(s) == 21  # one token once the whole prompt is in


def test_several_prompts_share_a_prefill_step(make_seq, make_config):
    sched = Scheduler(make_config())
    seqs = [make_seq(range(1, 4 + i)) for i in range(3)]
    for s in seqs:
        sched.add(s)
    got, pre = sched.schedule()
    assert pre and got == seqs


def test_max_num_seqs_caps_a_step(make_seq, make_config):
    sched = Scheduler(make_config(max_num_seqs=2))
    for i in range(3):
        sched.add(make_seq(range(1, 5)))
    got, _ = sched.schedule()
    assert len(got) == 2


def test_a_prompt_that_does_not_fit_waits_for_the_next_step(make_seq, make_config):
    sched = Scheduler(make_config(max_num_batched_tokens=10))
    a, b = make_seq(range(1, 7)), make_seq(range(1, 9))
    sched.add(a)
    sched.add(b)
    got, _ = sched.schedule()
    assert got == [a] and b.block_table == []  # only the first prompt of a step is ever chunked


def test_block_exhaustion_preempts_the_newest_running_sequence(make_seq, make_config):
    sched = Scheduler(make_config(num_kvcache_blocks=4))
    a, b = make_seq(range(1, 5), ignore_eos=True), make_seq(range(11, 15), ignore_eos=True)
    sched.add(a)
    sched.add(b)
    _step(sched)  # both prefilled: one full block each
    _step(sched)  # decode: each takes its second block (pool now empty)
    _step(sched)
    _step(sched)
    _step(sched)  # lengths reach 8 (second block full)
    got, pre = sched.schedule()  # a needs a third block: b is preempted
    assert not pre and got == [a] and b.status == SequenceStatus.WAITING and b.block_table == []
    assert sched.waiting[0] is b


def test_eos_finishes_a_sequence_unless_ignored(make_seq, make_config):
    sched = Scheduler(make_config(eos=2))
    stop, go = make_seq(range(3, 6)), make_seq(range(3, 6), ignore_eos=True)
    sched.add(stop)
    sched.add(go)
    _step(sched, token=2)
    assert stop.status == SequenceStatus.FINISHED and go.status == SequenceStatus.RUNNING


def test_max_tokens_finishes_a_sequence(make_seq, make_config):
    sched = Scheduler(make_config())
    s = make_seq(range(3, 6), max_tokens=2, ignore_eos=True)
    sched.add(s)
    _step(sched)
    assert s.status == SequenceStatus.RUNNING
    _step(sched)
    assert s.status == SequenceStatus.FINISHED and s.completion_token_ids == [7, 7]


# ------------------------------------------------------------------ ModelRunner
def test_runner_forwards_run_under_inference_mode():
    """Every ModelRunner method that runs the model (set-up forwards, graph
    capture, the step) is wrapped in torch.inference_mode: the buffers these
    create are inference tensors, and an in-place update of one outside
    inference mode (the sampler seed restore after capture) raises."""
    from kavor_b200.engine.model_runner import ModelRunner
    for name in ("_profile_prefill", "_profile_decode", "capture_cudagraph", "run_step", "run_async_step"):
        assert hasattr(getattr(ModelRunner, name), "__wrapped__"), name


class _FakePending:
    def __init__(self, tokens):
        self.tokens = tokens

    def result(self):
        return list(self.tokens)


class _FakeRunner:
    """Host model of ModelRunner.run / run_async: the 'device' samples
    (31 x input token + position) mod 1000; a chained step takes its input
    tokens from the previous step's samples, never from the host."""

    def __init__(self):
        self.device_sampled = None

    @staticmethod
    def _sample(inputs, positions):
        return [(31 * t + p) % 1000 for t, p in zip(inputs, positions)]

    def run(self, seqs, is_prefill):
        return self._sample([s.last_token for s in seqs], [len(s) - 1 for s in seqs])

    def run_async(self, seqs, chain=False):
        inputs = self.device_sampled if chain else [s.last_token for s in seqs]
        assert all(t >= 0 for t in inputs), "a placeholder reached the model"
        self.device_sampled = self._sample(inputs, [len(s) - 1 for s in seqs])
        return _FakePending(self.device_sampled)


@pytest.mark.parametrize("steps", [1, 2, 7])
def test_pipelined_decode_ends_like_the_synchronous_one(make_seq, steps):
    """advance_decode with one step in flight (placeholders patched on read,
    inputs chained on the device) leaves every sequence, block table and
    cached-token count exactly as the step-by-step loop does."""
    from kavor_b200.engine.model_runner import advance_decode

    runs = []
    for pipelined in (False, True):
        bm = BlockManager(64, BS)
        seqs = [make_seq(range(10 + i, 13 + 2 * i)) for i in range(3)]
        for s in seqs:
            bm.allocate_prefill(s, 0)
            s.num_cached_tokens = len(s)
        advance_decode(_FakeRunner(), seqs, bm, steps, pipelined=pipelined)
        runs.append([(s.token_ids, s.last_token, s.block_table, s.num_cached_tokens, len(s)) for s in seqs])
    assert runs[0] == runs[1]


class _FakeEngineRunner:
    """Host model of the runner behind the engine: the 'device' samples
    (7 x input token + 13 x position) mod 50 for every step, prefill chunks
    included; token 3 is the end of sequence. run_async keeps its samples on
    the 'device' and a chained step reads its inputs from them (row map or
    same order), never from the host's placeholder."""

    VOCAB = 50

    def __init__(self):
        self.device_sampled = None

    def _tok(self, inp, pos):
        return (7 * inp + 13 * pos) % self.VOCAB

    def call(self, method, *args):
        return getattr(self, method)(*args)

    def run(self, seqs, is_prefill):
        if is_prefill:
            ends = [s.num_cached_tokens + s.num_scheduled_tokens - 1 for s in seqs]
            return [self._tok(s.token_ids[e], e) for s, e in zip(seqs, ends)]
        return [self._tok(s.last_token, len(s) - 1) for s in seqs]

    def run_async(self, seqs, chain=False):
        if chain is True:
            inputs = list(self.device_sampled)
        elif chain:
            inputs = [self.device_sampled[i] for i in chain]
        else:
            inputs = [s.last_token for s in seqs]
        assert all(t >= 0 for t in inputs), "a placeholder reached the model"
        self.device_sampled = [self._tok(t, len(s) - 1) for t, s in zip(inputs, seqs)]
        return _FakePending(self.device_sampled)


def _engine_outputs(make_config, make_seq, pipelined, num_blocks, arrivals):
    from kavor_b200.engine.pipeline import DecodePipeline

    sched = Scheduler(make_config(eos=3, num_kvcache_blocks=num_blocks, max_num_batched_tokens=24, max_num_seqs=6))
    runner = _FakeEngineRunner()
    pipe = DecodePipeline(sched, runner.call) if pipelined else None
    finished, step = {}, 0
    pending = list(arrivals)
    while pending or not (pipe.is_finished() if pipe else sched.is_finished()):
        while pending and pending[0][0] <= step:  # requests arriving while others run
            _, prompt, max_tokens, ignore_eos = pending.pop(0)
            sched.add(make_seq(prompt, max_tokens=max_tokens, ignore_eos=ignore_eos))
        step += 1
        if pipe is not None:
            done = pipe.step()
        else:
            if sched.is_finished():
                continue
            seqs, is_prefill = sched.schedule()
            sched.postprocess(seqs, runner.run(seqs, is_prefill), is_prefill)
            done = [s for s in seqs if s.is_finished]
        for s in done:
            assert s.seq_id not in finished
            finished[s.seq_id] = (s.prompt_token_ids, s.completion_token_ids)
    bm = sched.block_manager
    assert len(bm.free_block_ids) == num_blocks and not bm.used_block_ids
    return sorted(finished.values())


@pytest.mark.parametrize("num_blocks", [64, 12])  # 12 blocks of 4 tokens: decode preempts
def test_decode_pipeline_gives_the_step_at_a_time_outputs(make_seq, make_config, num_blocks):
    """DecodePipeline (one decode step in flight, placeholders, tokens chained
    on the device, end-of-sequence seen one step late) returns exactly the
    completions of the schedule -> run -> postprocess loop: prompts of
    different lengths (chunked prefill), max_tokens and end-of-sequence
    finishes, requests arriving mid-run, and a pool small enough to preempt."""
    arrivals = [(0, [5, 9, 11, 2, 8, 30], 9, False), (0, list(range(1, 20)), 14, False), (0, [4], 6, True),
                (0, [17, 17, 17, 17, 17], 20, False), (3, [6, 7], 5, False), (9, list(range(21, 31)), 11, True),
                (9, [12, 1, 44], 25, False), (15, [2], 7, False)]
    sync = _engine_outputs(make_config, make_seq, False, num_blocks, arrivals)
    piped = _engine_outputs(make_config, make_seq, True, num_blocks, arrivals)
    assert piped == sync
    assert any(c and c[-1] == 3 for _, c in sync)  # some sequence ended on its end-of-sequence token


def test_shared_prefix_workload_shape():
    """The prefill-heavy benchmark's prompts: one shared 2048-token prefix,
    unique suffixes of U[512, 6144] tokens, ids in [0, 10000], reproducible."""
    from kavor_b200.bench_prefix import workload

    prompts = workload(64, 2048, 512, 6144)
    assert len(prompts) == 64 and prompts == workload(64, 2048, 512, 6144)
    prefix = prompts[0][:2048]
    assert all(p[:2048] == prefix and 512 <= len(p) - 2048 <= 6144 for p in prompts)
    assert all(0 <= t <= 10000 for p in prompts for t in p)
    assert len({tuple(p[2048:2060]) for p in prompts}) == 64


def test_profile_host_runs(capsys):
    """The host-step profile (schedule, metadata, postprocess, TP message
    forms, pipelined step) runs on the CPU and reports every field."""
    import json

    from kavor_b200 import profile_host

    assert profile_host.main(["--batch", "8", "--context", "300", "--steps", "5"]) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    for k in ("schedule", "metadata", "postprocess", "tp_message_sequences", "tp_message_metadata", "pipeline_step"):
        assert line[k] > 0, k
