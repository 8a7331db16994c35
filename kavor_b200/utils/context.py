"""Per-step forward metadata read by the attention layers.

Same fields and semantics as the reference's global context
(kavor/utils/context.py:5-32) for full-attention models: ``is_prefill``,
``cu_seqlens_q/k`` (int32 [B+1]), ``max_seqlen_q/k``, ``slot_mapping`` (int32
[T], -1 = padding), ``context_lens`` (int32 [B]) and ``block_tables`` (int32
[B, max_blocks], -1 padded; for prefill only when a prefix is cached).
"""
from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass

import torch


@dataclass(slots=True)
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(is_prefill: bool, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q: int = 0,
                max_seqlen_k: int = 0, slot_mapping=None, context_lens=None, block_tables=None) -> None:
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping,
                       context_lens, block_tables)


def reset_context() -> None:
    global _CONTEXT
    _CONTEXT = Context()


@contextmanager
def context_scope(ctx: Context):
    """Make `ctx` the current context inside the block (the one before it is
    restored on exit): a decode step split into row ranges gives each range
    the slices of the step's metadata."""
    global _CONTEXT
    prev, _CONTEXT = _CONTEXT, ctx
    try:
        yield ctx
    finally:
        _CONTEXT = prev


def decode_rows(ctx: Context, lo: int, hi: int) -> Context:
    """The decode context of rows [lo, hi) of a decode step's context."""
    if ctx.is_prefill:
        raise ValueError("decode_rows: prefill contexts are not split by rows")
    return Context(False, slot_mapping=ctx.slot_mapping[lo:hi], context_lens=ctx.context_lens[lo:hi],
                   block_tables=ctx.block_tables[lo:hi])
