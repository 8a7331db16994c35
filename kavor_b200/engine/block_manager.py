"""KV block allocator with prefix caching (drop-in for kavor/engine/block_manager.py,
full-attention path).

Allocation order, reuse and eviction follow block_manager.py:40-243 exactly so
block tables (and therefore slot mappings) are identical to the reference's:

* free blocks form a FIFO (``popleft`` to allocate, ``append`` to free);
* a full block is keyed by a chained hash of (parent block hash, its tokens);
  a prompt reuses its leading full blocks (never its last block) while the
  chain hits and the stored tokens match;
* a reused block that is still referenced only gains a reference, a freed one
  is taken back out of the free list; a freed block keeps its hash until it is
  handed out again (lazy eviction).

The chained key is SHA-256 over the parent key and the token ids as int64
little-endian bytes; only equality of keys matters to the allocator.
"""
from __future__ import annotations

import hashlib
from collections import deque

import numpy as np

from kavor_b200.engine.sequence import Sequence

NONE_HASH = b""


class Block:

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash: bytes | int = -1
        self.token_ids: list[int] = []

    def update(self, h: bytes, token_ids: list[int]) -> None:
        self.hash = h
        self.token_ids = token_ids

    def reset(self) -> None:
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []


class BlockManager:

    def __init__(self, num_blocks: int, block_size: int, enable_prefix_cache: bool = True):
        if num_blocks <= 0:
            raise ValueError("the KV pool needs at least one block")
        self.block_size = block_size
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[bytes, int] = {}
        self.free_block_ids: deque[int] = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()
        self.enable_prefix_cache = enable_prefix_cache
        self.prefix_cache_hit_tokens = 0
        self.prefix_cache_prompt_tokens = 0

    @staticmethod
    def hash_block_tokens(parent: bytes | int, token_ids: list[int]) -> bytes:
        h = hashlib.sha256()
        h.update(parent if isinstance(parent, bytes) else NONE_HASH)
        h.update(np.asarray(token_ids, dtype="<i8").tobytes())
        return h.digest()

    def allocate_block(self) -> int:
        block_id = self.free_block_ids.popleft()
        block = self.blocks[block_id]
        assert block.ref_count == 0
        if block.hash != -1 and self.hash_to_block_id.get(block.hash) == block_id:
            del self.hash_to_block_id[block.hash]
        block.reset()
        self.used_block_ids.add(block_id)
        return block_id

    def deallocate_block(self, block_id: int) -> None:
        assert self.blocks[block_id].ref_count == 0
        self.used_block_ids.remove(block_id)
        self.free_block_ids.append(block_id)

    def can_allocate_prefill(self, seq: Sequence) -> tuple[int, None]:
        """(number of leading blocks served from the prefix cache, None), or
        (-1, None) when the free list cannot hold the rest."""
        num_cached = 0
        needed = seq.num_blocks
        if self.enable_prefix_cache:
            parent: bytes | int = -1
            for i in range(seq.num_blocks - 1):
                tokens = seq.block(i)
                parent = self.hash_block_tokens(parent, tokens)
                block_id = self.hash_to_block_id.get(parent, -1)
                if block_id == -1 or self.blocks[block_id].token_ids != tokens:
                    break
                num_cached += 1
                if block_id in self.used_block_ids:
                    needed -= 1
        if len(self.free_block_ids) < needed:
            return -1, None
        return num_cached, None

    def allocate_prefill(self, seq: Sequence, num_cached_blocks: int, bundle=None) -> None:
        assert not seq.block_table
        parent: bytes | int = -1
        for i in range(num_cached_blocks):
            tokens = seq.block(i)
            parent = self.hash_block_tokens(parent, tokens)
            block_id = self.hash_to_block_id[parent]
            block = self.blocks[block_id]
            if block_id in self.used_block_ids:
                block.ref_count += 1
            else:
                block.ref_count = 1
                self.free_block_ids.remove(block_id)
                self.used_block_ids.add(block_id)
            seq.block_table.append(block_id)
        for _ in range(num_cached_blocks, seq.num_blocks):
            seq.block_table.append(self.allocate_block())
        cached_tokens = num_cached_blocks * self.block_size
        seq.num_cached_tokens = cached_tokens
        if self.enable_prefix_cache:
            self.prefix_cache_hit_tokens += cached_tokens
            self.prefix_cache_prompt_tokens += seq.num_tokens

    def deallocate(self, seq: Sequence) -> None:
        for block_id in reversed(seq.block_table):
            block = self.blocks[block_id]
            block.ref_count -= 1
            if block.ref_count == 0:
                self.deallocate_block(block_id)
        seq.num_cached_tokens = 0
        seq.block_table.clear()

    def can_append_block(self, seq: Sequence) -> bool:
        return len(self.free_block_ids) >= (seq.num_tokens % self.block_size == 1)

    def may_append_block(self, seq: Sequence) -> None:
        if seq.num_tokens % self.block_size == 1:
            seq.block_table.append(self.allocate_block())

    def may_append_blocks(self, seqs: list[Sequence]) -> None:
        """may_append_block for every sequence of a decode batch, in order (one
        Python frame for the batch: this runs on the host every decode step)."""
        bs = self.block_size
        for seq in seqs:
            if seq.num_tokens % bs == 1:
                seq.block_table.append(self.allocate_block())

    def hash_blocks(self, seq: Sequence) -> None:
        """Key every block completed by this step so later prompts can reuse it."""
        if not self.enable_prefix_cache:
            return
        start = seq.num_cached_tokens // self.block_size
        end = (seq.num_cached_tokens + seq.num_scheduled_tokens) // self.block_size
        if start == end:
            return
        parent = self.blocks[seq.block_table[start - 1]].hash if start > 0 else -1
        for i in range(start, end):
            block = self.blocks[seq.block_table[i]]
            tokens = seq.block(i)
            parent = self.hash_block_tokens(parent, tokens)
            block.update(parent, tokens)
            self.hash_to_block_id[parent] = block.block_id
