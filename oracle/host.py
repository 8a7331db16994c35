"""Host batch metadata, restated as the reference's own loops (test infrastructure).

prepare_prefill: model_runner.py:385-446 (slot ranges walked block by block,
:418-430); prepare_decode: model_runner.py:448-467; block tables padded with
-1: model_runner.py:469-473. Sequences are any objects with the Sequence
fields (token_ids, num_cached_tokens, num_scheduled_tokens, block_table,
last_token, num_tokens).
"""
from __future__ import annotations


def block_tables(seqs) -> list[list[int]]:
    width = max(len(s.block_table) for s in seqs)
    return [list(s.block_table) + [-1] * (width - len(s.block_table)) for s in seqs]


def prepare_prefill(seqs, block_size: int) -> dict:
    input_ids, positions, slot_mapping = [], [], []
    cu_q, cu_k = [0], [0]
    max_q = max_k = 0
    for s in seqs:
        start = s.num_cached_tokens
        end = start + s.num_scheduled_tokens
        input_ids.extend(s.token_ids[start:end])
        positions.extend(range(start, end))
        cu_q.append(cu_q[-1] + end - start)
        cu_k.append(cu_k[-1] + end)
        max_q = max(max_q, end - start)
        max_k = max(max_k, end)
        if not s.block_table:
            continue
        first, last = start // block_size, (end + block_size - 1) // block_size
        for i in range(first, last):
            lo = s.block_table[i] * block_size + (start % block_size if i == first else 0)
            if i != last - 1:
                hi = s.block_table[i] * block_size + block_size
            else:
                hi = s.block_table[i] * block_size + end - i * block_size
            slot_mapping.extend(range(lo, hi))
    return {
        "input_ids": input_ids, "positions": positions, "cu_seqlens_q": cu_q, "cu_seqlens_k": cu_k,
        "max_seqlen_q": max_q, "max_seqlen_k": max_k, "slot_mapping": slot_mapping,
        "block_tables": block_tables(seqs) if cu_k[-1] > cu_q[-1] else None,
    }


def prepare_decode(seqs, block_size: int) -> dict:
    return {
        "input_ids": [s.last_token for s in seqs],
        "positions": [s.num_tokens - 1 for s in seqs],
        # last_block_num_tokens = num_tokens - (num_blocks - 1) * block_size (sequence.py:573-575)
        "slot_mapping": [s.block_table[-1] * block_size
                         + s.num_tokens - ((s.num_tokens + block_size - 1) // block_size - 1) * block_size - 1
                         for s in seqs],
        "context_lens": [s.num_tokens for s in seqs],
        "block_tables": block_tables(seqs),
    }
