"""Host-side cost of one engine step (no GPU needed).

    python -m kavor_b200.profile_host [--batch 256 --context 1000 --steps 200]

B sequences of `context` random prompt tokens are prefilled through the
Scheduler (block size 256, prefix caching off, ignore_eos), then decode
steps run with a stand-in for the model that returns a fixed token, so
only the host's share of a step is timed (time.perf_counter, mean over
`steps`):

* ``schedule``: Scheduler.schedule (block growth included);
* ``metadata``: decode_metadata (ids, positions, slots, context lengths and
  the padded block-table matrix);
* ``postprocess``: Scheduler.postprocess;
* ``tp_message_sequences``: pickling the step's sequences, as a mailbox
  message that carried them (model_runner.py:93-112 of the reference), and
  ``tp_unpickle_sequences`` + ``metadata`` on a worker;
* ``tp_message_metadata``: pickling the metadata arrays that
  ModelRunner.call sends instead, and ``tp_unpickle_metadata`` on a worker;
* ``pipeline_step``: DecodePipeline.step (schedule + provisional + finalize).

Prints one JSON line of microseconds per step.
"""
from __future__ import annotations

import argparse
import json
import pickle
import random
import time
from types import SimpleNamespace

import numpy as np


def _mean_us(fn, n: int) -> float:
    t0 = time.perf_counter()
    for _ in range(n):
        fn()
    return (time.perf_counter() - t0) / n * 1e6


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--context", type=int, default=1000)
    ap.add_argument("--steps", type=int, default=200)
    a = ap.parse_args(argv)

    from kavor_b200.engine.model_runner import decode_metadata
    from kavor_b200.engine.pipeline import DecodePipeline
    from kavor_b200.engine.scheduler import Scheduler
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    bs = 256
    Sequence.block_size = bs  # as ModelRunner sets it from the config
    blocks_per_seq = (a.context + 3 * a.steps) // bs + 2
    cfg = SimpleNamespace(max_num_seqs=a.batch, max_num_batched_tokens=max(16384, a.context), eos=-1,
                          kvcache_block_size=bs, num_kvcache_blocks=a.batch * blocks_per_seq,
                          enable_prefix_caching=False)
    random.seed(0)
    sched = Scheduler(cfg)
    params = SamplingParams(temperature=0.6, max_tokens=1 << 30, ignore_eos=True)
    for _ in range(a.batch):
        sched.add(Sequence([random.randint(0, 10000) for _ in range(a.context)], params))
    while sched.waiting:
        seqs, is_prefill = sched.schedule()
        sched.postprocess(seqs, [1] * len(seqs), is_prefill)

    t = {"schedule": 0.0, "metadata": 0.0, "postprocess": 0.0}
    for _ in range(a.steps):
        t0 = time.perf_counter()
        seqs, _ = sched.schedule()
        t1 = time.perf_counter()
        decode_metadata(seqs, bs)
        t2 = time.perf_counter()
        sched.postprocess(seqs, [5] * len(seqs), False)
        t3 = time.perf_counter()
        t["schedule"] += t1 - t0
        t["metadata"] += t2 - t1
        t["postprocess"] += t3 - t2
    out = {k: v / a.steps * 1e6 for k, v in t.items()}

    seqs, _ = sched.schedule()
    meta = decode_metadata(seqs, bs)
    temps = np.fromiter((s.temperature for s in seqs), np.float32, len(seqs))
    msg_seqs = pickle.dumps(["run", seqs, False])
    msg_meta = pickle.dumps(["run_step", meta, temps, False])
    out["tp_message_sequences"] = _mean_us(lambda: pickle.dumps(["run", seqs, False]), a.steps)
    out["tp_unpickle_sequences"] = _mean_us(lambda: pickle.loads(msg_seqs), a.steps)
    out["tp_message_metadata"] = _mean_us(lambda: pickle.dumps(["run_step", meta, temps, False]), a.steps)
    out["tp_unpickle_metadata"] = _mean_us(lambda: pickle.loads(msg_meta), a.steps)
    out["tp_message_bytes"] = {"sequences": len(msg_seqs), "metadata": len(msg_meta)}
    sched.postprocess(seqs, [5] * len(seqs), False)

    class _Done:
        def __init__(self, n):
            self.n = n

        def result(self):
            return [5] * self.n

    pipe = DecodePipeline(sched, lambda method, seqs, chain: _Done(len(seqs)))
    out["pipeline_step"] = _mean_us(pipe.step, a.steps)
    rounded = {k: (round(v, 1) if isinstance(v, float) else v) for k, v in out.items()}
    print(json.dumps({"workload": f"decode host step, B={a.batch}, context {a.context}, block 256",
                      "unit": "us per step", **rounded}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
