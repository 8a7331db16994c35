"""Sequence state (drop-in for kavor/engine/sequence.py, text-only).

A sequence owns its token ids, its logical->physical block table and the
scheduling counters the block manager and model runner read
(``num_cached_tokens``: tokens whose KV is in the cache, ``num_scheduled_tokens``:
tokens computed in the current step). Pickling for TP workers sends the full
token list during prefill and only the last token during decode
(sequence.py:602-618), keeping the per-step message small.
"""
from __future__ import annotations

from copy import copy
from dataclasses import dataclass, field
from enum import Enum, auto
from itertools import count
from time import perf_counter

from kavor_b200.sampling_params import SamplingParams


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


@dataclass
class SeqStats:
    """Per-request timing and prefix-cache statistics (engine side only)."""

    arrival_time: float = field(default_factory=perf_counter)
    prefill_start_time: float | None = None
    first_token_time: float | None = None
    finish_time: float | None = None
    prefix_cache_hit_tokens: int | None = None

    def mark_prefill_start(self) -> None:
        if self.prefill_start_time is None:
            self.prefill_start_time = perf_counter()

    def record_prefix_cache(self, hit_tokens: int) -> None:
        if self.prefix_cache_hit_tokens is None:
            self.prefix_cache_hit_tokens = hit_tokens


class Sequence:
    block_size = 256
    counter = count()

    def __init__(self, inputs, sampling_params: SamplingParams = SamplingParams()):
        token_ids = getattr(inputs, "token_ids", inputs)
        if not len(token_ids):
            raise ValueError("a sequence needs at least one prompt token")
        self.seq_id = next(Sequence.counter)
        self.status = SequenceStatus.WAITING
        self.token_ids = list(copy(token_ids))
        self.last_token = self.token_ids[-1]
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = self.num_tokens
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.is_prefill = True
        self.block_table: list[int] = []
        self.temperature = sampling_params.temperature
        self.max_tokens = sampling_params.max_tokens
        self.ignore_eos = sampling_params.ignore_eos
        self.request_id: str | None = None
        self.stats: SeqStats | None = SeqStats()

    def __len__(self) -> int:
        return self.num_tokens

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def prompt_token_ids(self) -> list[int]:
        return self.token_ids[:self.num_prompt_tokens]

    @property
    def completion_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_blocks(self) -> int:
        return (self.num_tokens + self.block_size - 1) // self.block_size

    @property
    def last_block_num_tokens(self) -> int:
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    def block(self, i: int) -> list[int]:
        if not 0 <= i < self.num_blocks:
            raise IndexError(f"block {i} out of range [0, {self.num_blocks})")
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(token_id)
        self.last_token = token_id
        self.num_tokens += 1

    def __getstate__(self):
        tokens = self.token_ids if self.is_prefill else self.last_token
        return (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
                self.num_scheduled_tokens, self.block_table, tokens, self.temperature, self.is_prefill)

    def __setstate__(self, state):
        (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens, self.num_scheduled_tokens,
         self.block_table, tokens, self.temperature, self.is_prefill) = state
        self.stats = None
        if isinstance(tokens, list):
            self.token_ids = tokens
            self.last_token = tokens[-1]
        else:
            self.token_ids = []
            self.last_token = tokens
