"""Engine steps with one decode step in flight (no reference counterpart: the
reference's engine loop, llm_engine.py:245-272, runs schedule -> run ->
postprocess one step at a time, so the GPU waits while the host schedules).

``DecodePipeline.step()`` issues decode step i+1 through
``ModelRunner.run_async`` before it reads step i's tokens: step i+1's input
tokens are step i's samples, gathered on the device (the chain map gives each
sequence its row in step i's batch). To schedule step i+1 without step i's
tokens, every sequence of step i is advanced on the host right after the
issue with a placeholder token (``provisional``) and patched when the tokens
arrive (``finalize``):

* a sequence that reaches ``max_tokens`` finishes at once (it is not
  scheduled again; it is reported when its last token arrives);
* an end-of-sequence token is only seen at finalize, after the sequence was
  scheduled into the next step: it finishes then, and its token from that
  next step is dropped;
* prefill steps run as before, synchronously, after the decode step in flight
  has been finalized;
* the prefix-cache key of a block is computed when the token that completes
  it is known (hash_blocks runs in provisional on the step's input tokens,
  which finalize of the step before has already patched).

Tokens, block tables and finish order equal those of the one-step-at-a-time
loop for the same sampler outputs (tests/test_engine_host.py).
"""
from __future__ import annotations

from dataclasses import dataclass

from kavor_b200.engine.sequence import Sequence, SequenceStatus

PLACEHOLDER = -1


@dataclass
class _InFlight:
    seqs: list[Sequence]
    pending: object           # PendingDecode (result() -> list[int])
    live: list[bool]          # the sequences this step's tokens belong to


class DecodePipeline:

    def __init__(self, scheduler, call):
        self.scheduler = scheduler
        self.call = call          # call(method, *args): the model runner's dispatch (TP mailbox included)
        self.inflight: _InFlight | None = None

    def is_finished(self) -> bool:
        return self.inflight is None and self.scheduler.is_finished()

    def step(self) -> list[Sequence]:
        """Advance by one issued step (or one drain); returns the sequences
        whose tokens became final and that finished."""
        sched = self.scheduler
        fl = self.inflight
        if fl is None:
            seqs, is_prefill = sched.schedule()
            if is_prefill:
                token_ids = self.call("run", seqs, True)
                sched.postprocess(seqs, token_ids, True)
                return [s for s in seqs if s.is_finished]
            pending = self.call("run_async", seqs, False)
            self.inflight = _InFlight(seqs, pending, self._provisional(seqs))
            return []
        if sched.waiting or not sched.running:
            return self._finalize(fl)  # a prefill (or nothing) comes next: no step to chain
        rows = {id(s): i for i, s in enumerate(fl.seqs)}
        seqs, is_prefill = sched.schedule()
        assert not is_prefill  # nothing was waiting
        if any(id(s) not in rows for s in seqs):  # not a sub-batch of the step in flight: start over
            done = self._finalize(fl)
            pending = self.call("run_async", seqs, False)
            self.inflight = _InFlight(seqs, pending, self._provisional(seqs))
            return done
        chain = [rows[id(s)] for s in seqs]
        pending = self.call("run_async", seqs, True if chain == list(range(len(fl.seqs))) else chain)
        done = self._finalize(fl)
        self.inflight = _InFlight(seqs, pending, self._provisional(seqs))
        return done

    def _provisional(self, seqs: list[Sequence]) -> list[bool]:
        """Scheduler.postprocess for a step whose tokens are not known yet."""
        sched, bm = self.scheduler, self.scheduler.block_manager
        live = []
        for seq in seqs:
            if seq.is_finished:  # an end-of-sequence token of the step before: this step is void for it
                live.append(False)
                continue
            bm.hash_blocks(seq)
            seq.num_cached_tokens += seq.num_scheduled_tokens
            seq.num_scheduled_tokens = 0
            seq.append_token(PLACEHOLDER)
            if seq.num_completion_tokens == seq.max_tokens:
                seq.status = SequenceStatus.FINISHED
                bm.deallocate(seq)
                sched.running.remove(seq)
            live.append(True)
        return live

    def _finalize(self, fl: _InFlight) -> list[Sequence]:
        sched = self.scheduler
        done = []
        for seq, tok, live in zip(fl.seqs, fl.pending.result(), fl.live):
            if not live:
                continue
            seq.token_ids[-1] = seq.last_token = tok
            if seq.is_finished:  # max_tokens, decided in provisional
                done.append(seq)
            elif not seq.ignore_eos and tok == sched.eos:
                if seq.status == SequenceStatus.WAITING:  # preempted since: no blocks held
                    sched.waiting.remove(seq)
                else:
                    sched.block_manager.deallocate(seq)
                    sched.running.remove(seq)
                seq.status = SequenceStatus.FINISHED
                done.append(seq)
        self.inflight = None
        return done
