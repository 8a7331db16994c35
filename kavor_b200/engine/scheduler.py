"""Prefill-first scheduler with chunked prefill and preemption
(drop-in for kavor/engine/scheduler.py, full-attention path: scheduler.py:100-190).

* A step is either all prefill or all decode. Prefill takes waiting
  sequences in FIFO order under ``max_num_batched_tokens`` (a sequence that
  does not fit is chunked only if it is the first of the step) and
  ``max_num_seqs``.
* Decode takes running sequences in order; when a sequence needs a new block
  and none is free, the most recently added running sequence is preempted
  (its blocks freed, back to the head of the waiting queue), or the sequence
  itself if it is the last one.
"""
from __future__ import annotations

from collections import deque

from kavor_b200.engine.block_manager import BlockManager
from kavor_b200.engine.sequence import Sequence, SequenceStatus


class Scheduler:

    def __init__(self, config):
        self.config = config
        self.max_num_seqs = config.max_num_seqs
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.eos = config.eos
        self.block_size = config.kvcache_block_size
        self.block_manager = BlockManager(config.num_kvcache_blocks, config.kvcache_block_size,
                                          enable_prefix_cache=getattr(config, "enable_prefix_caching", True))
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence) -> None:
        self.waiting.append(seq)

    def schedule(self) -> tuple[list[Sequence], bool]:
        scheduled: list[Sequence] = []
        batched = 0
        bm = self.block_manager
        while self.waiting and len(scheduled) < self.max_num_seqs:
            seq = self.waiting[0]
            remaining = self.max_num_batched_tokens - batched
            if remaining == 0:
                break
            if not seq.block_table:
                num_cached_blocks, _ = bm.can_allocate_prefill(seq)
                if num_cached_blocks == -1:
                    break
                num_tokens = seq.num_tokens - num_cached_blocks * self.block_size
            else:
                num_tokens = seq.num_tokens - seq.num_cached_tokens
            if remaining < num_tokens and scheduled:
                break
            if not seq.block_table:
                bm.allocate_prefill(seq, num_cached_blocks)
                if seq.stats is not None:
                    seq.stats.mark_prefill_start()
                    if bm.enable_prefix_cache:
                        seq.stats.record_prefix_cache(seq.num_cached_tokens)
            seq.num_scheduled_tokens = min(num_tokens, remaining)
            batched += seq.num_scheduled_tokens
            if seq.num_cached_tokens + seq.num_scheduled_tokens == seq.num_tokens:
                seq.status = SequenceStatus.RUNNING
                self.waiting.popleft()
                self.running.append(seq)
            scheduled.append(seq)
        if scheduled:
            return scheduled, True

        while self.running and len(scheduled) < self.max_num_seqs:
            seq = self.running.popleft()
            while not bm.can_append_block(seq):
                if self.running:
                    self.preempt(self.running.pop())
                else:
                    self.preempt(seq)
                    break
            else:
                seq.num_scheduled_tokens = 1
                seq.is_prefill = False
                bm.may_append_block(seq)
                scheduled.append(seq)
        if not scheduled:
            raise RuntimeError("nothing to schedule: the KV pool cannot hold a single running sequence")
        self.running.extendleft(reversed(scheduled))
        return scheduled, False

    def preempt(self, seq: Sequence) -> None:
        seq.status = SequenceStatus.WAITING
        seq.is_prefill = True
        self.block_manager.deallocate(seq)
        self.waiting.appendleft(seq)

    def postprocess(self, seqs: list[Sequence], token_ids: list[int], is_prefill: bool) -> None:
        for seq, token_id in zip(seqs, token_ids):
            self.block_manager.hash_blocks(seq)
            seq.num_cached_tokens += seq.num_scheduled_tokens
            seq.num_scheduled_tokens = 0
            if is_prefill and seq.num_cached_tokens < seq.num_tokens:
                continue  # chunk of a longer prompt: no token yet
            seq.append_token(token_id)
            if (not seq.ignore_eos and token_id == self.eos) or seq.num_completion_tokens == seq.max_tokens:
                seq.status = SequenceStatus.FINISHED
                self.block_manager.deallocate(seq)
                self.running.remove(seq)
