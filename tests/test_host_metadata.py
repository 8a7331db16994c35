"""Host-side parity: scheduling, block tables, slot mappings and batch metadata
must be bit-exact with the reference (tests/golden/host_trace.json was
recorded from the reference's Scheduler/BlockManager/ModelRunner)."""
import json
import random
from types import SimpleNamespace

import numpy as np
import pytest

import cases
from conftest import GOLDEN
from oracle import host as ohost


def _golden():
    return json.loads((GOLDEN / "host_trace.json").read_text())


def _run_product(meta_source: str):
    from kavor_b200.engine.model_runner import decode_metadata, prefill_metadata
    from kavor_b200.engine.scheduler import Scheduler
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    _, _, _, cfg = cases.host_workload()
    bs = cfg["kvcache_block_size"]
    sched = Scheduler(SimpleNamespace(**cfg))

    def make_seq(prompt, p):
        return Sequence(list(prompt), SamplingParams(temperature=1.0, max_tokens=p[0], ignore_eos=p[1]))

    if meta_source == "product":
        mp = lambda seqs: prefill_metadata(seqs, bs)  # noqa: E731
        md = lambda seqs: decode_metadata(seqs, bs)  # noqa: E731
    else:
        mp = lambda seqs: ohost.prepare_prefill(seqs, bs)  # noqa: E731
        md = lambda seqs: ohost.prepare_decode(seqs, bs)  # noqa: E731
    trace, final = cases.run_host_trace(make_seq, sched, mp, md)
    return trace, final, sched.block_manager


@pytest.mark.parametrize("source", ["product", "oracle"])
def test_trace_is_bit_exact_with_reference(source):
    gold = _golden()
    trace, final, bm = _run_product(source)
    assert len(trace) == len(gold["trace"])
    for mine, ref in zip(trace, gold["trace"]):
        assert mine["step"] == ref["step"] and mine["prefill"] == ref["prefill"]
        assert mine["reqs"] == ref["reqs"], f"step {ref['step']}: scheduled requests differ"
        assert mine["tokens"] == ref["tokens"]
        for key, val in ref["meta"].items():
            assert mine["meta"][key] == val, f"step {ref['step']}: {key} differs"
    assert {str(k): v for k, v in final.items()} == gold["completions"]
    assert bm.prefix_cache_hit_tokens == gold["prefix_cache_hit_tokens"]
    assert bm.prefix_cache_prompt_tokens == gold["prefix_cache_prompt_tokens"]


def test_trace_exercises_prefix_hits_chunking_and_preemption():
    gold = _golden()
    assert gold["prefix_cache_hit_tokens"] > 0
    assert any(e["prefill"] and len(e["meta"]["input_ids"]) == 64 for e in gold["trace"])  # budget-limited chunk
    assert any(e["prefill"] and e["meta"]["block_tables"] is not None for e in gold["trace"])
    # a request that was prefilled, decoded, then scheduled for prefill again was preempted
    seen_decode, repeated = set(), False
    for e in gold["trace"]:
        if e["prefill"]:
            repeated |= bool(seen_decode & set(e["reqs"]))
        else:
            seen_decode |= set(e["reqs"])
    assert repeated


def test_vectorised_metadata_equals_reference_loops_on_random_states():
    """decode_metadata / prefill_metadata vs the reference's loop algorithm on
    random block tables, cached prefixes and chunk sizes (block_size 256)."""
    from kavor_b200.engine.model_runner import decode_metadata, prefill_metadata

    rng = random.Random(7)
    bs = 256
    for _ in range(50):
        seqs = []
        for _ in range(rng.randint(1, 8)):
            n = rng.randint(1, 3000)
            nb = (n + bs - 1) // bs
            cached = rng.randint(0, n - 1) // bs * bs if rng.random() < 0.5 else 0
            seqs.append(SimpleNamespace(token_ids=[rng.randint(0, 151935) for _ in range(n)], num_tokens=n,
                                        last_token=None, block_table=rng.sample(range(10000), nb),
                                        num_cached_tokens=cached, num_scheduled_tokens=rng.randint(1, n - cached),
                                        last_block_num_tokens=n - (nb - 1) * bs))
            seqs[-1].last_token = seqs[-1].token_ids[-1]
        a, b = prefill_metadata(seqs, bs), ohost.prepare_prefill(seqs, bs)
        for k in b:
            va = a[k].tolist() if isinstance(a[k], np.ndarray) else a[k]
            assert va == b[k], k
        for s in seqs:
            s.__len__ = None
        dseqs = [_Len(s) for s in seqs]
        a, b = decode_metadata(dseqs, bs), ohost.prepare_decode(dseqs, bs)
        for k in b:
            assert a[k].tolist() == b[k], k
        dtypes = {"input_ids": np.int64, "positions": np.int64, "slot_mapping": np.int32, "context_lens": np.int32,
                  "block_tables": np.int32}
        assert {k: a[k].dtype for k in dtypes} == {k: np.dtype(v) for k, v in dtypes.items()}


def test_decode_metadata_rejects_a_sequence_without_blocks():
    from kavor_b200.engine.model_runner import decode_metadata

    seqs = [SimpleNamespace(num_tokens=5, last_token=1, block_table=[3]),
            SimpleNamespace(num_tokens=2, last_token=1, block_table=[])]
    with pytest.raises(ValueError, match="needs a block"):
        decode_metadata(seqs, 256)
    empty = decode_metadata([], 256)
    assert all(v.shape[0] == 0 for v in empty.values())


class _Len(SimpleNamespace):
    def __init__(self, s):
        super().__init__(**vars(s))

    def __len__(self):
        return self.num_tokens
