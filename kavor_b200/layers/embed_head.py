"""Vocab-parallel embedding and LM head (drop-in for kavor/layers/embed_head.py).

``VocabParallelEmbedding`` looks up its vocab shard with one kernel that zeroes
out-of-shard rows, then all-reduces across ranks (embed_head.py:34-42).
``ParallelLMHead.forward`` keeps the reference contract (embed_head.py:56-66):
on prefill it keeps the last token of every sequence, computes the shard's
logits and gathers the full [B, vocab] rows on rank 0 (other ranks get None).
``ParallelLMHead.sample`` is the fused alternative used by the model runner:
every rank scores its own vocab shard and only (score, index) pairs cross
ranks, so no logits are gathered.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from kavor_b200 import _kernels as K
from kavor_b200.layers.linear import _tp, linear
from kavor_b200.utils.context import get_context


class VocabParallelEmbedding(nn.Module):

    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.tp_rank, self.tp_size = _tp()
        if num_embeddings % self.tp_size:
            raise ValueError("vocab size must be divisible by the tensor-parallel size")
        self.num_embeddings = num_embeddings
        self.num_embeddings_per_partition = num_embeddings // self.tp_size
        self.vocab_start_idx = self.num_embeddings_per_partition * self.tp_rank
        self.vocab_end_idx = self.vocab_start_idx + self.num_embeddings_per_partition
        self.weight = nn.Parameter(torch.empty(self.num_embeddings_per_partition, embedding_dim))
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        shard = param.data.size(0)
        param.data.copy_(loaded_weight.narrow(0, self.tp_rank * shard, shard))

    def forward(self, x: torch.Tensor, reduce: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
        y = K.embedding(x, self.weight, self.vocab_start_idx, self.vocab_end_idx, self.num_embeddings, out=out)
        if reduce and self.tp_size > 1:
            dist.all_reduce(y)
        return y


class ParallelLMHead(VocabParallelEmbedding):

    def __init__(self, num_embeddings: int, embedding_dim: int, bias: bool = False):
        if bias:
            raise ValueError("ParallelLMHead has no bias")
        super().__init__(num_embeddings, embedding_dim)

    def _last_tokens(self, x: torch.Tensor) -> torch.Tensor:
        ctx = get_context()
        if ctx.is_prefill:
            x = x[ctx.cu_seqlens_q[1:] - 1].contiguous()
        return x

    def forward(self, x: torch.Tensor):
        logits = linear(self._last_tokens(x), self.weight)
        if self.tp_size > 1:
            parts = [torch.empty_like(logits) for _ in range(self.tp_size)] if self.tp_rank == 0 else None
            dist.gather(logits, parts, 0)
            logits = torch.cat(parts, -1) if self.tp_rank == 0 else None
        return logits

    def sample(self, x: torch.Tensor, temperatures: torch.Tensor, seed: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """Logits of this shard and Gumbel-max over the full vocabulary without
        gathering logits; every rank returns the same token ids. Identical to
        ``Sampler()(forward(x), temperatures)`` with the same seed value."""
        logits = linear(self._last_tokens(x), self.weight)
        B = logits.shape[0]
        if out is None:
            out = torch.empty(B, dtype=torch.int64, device=logits.device)
        if self.tp_size == 1:
            return K.sample(logits, temperatures, seed, out=out)
        val = torch.empty(B, dtype=torch.float32, device=logits.device)
        idx = torch.empty(B, dtype=torch.int64, device=logits.device)
        K.sample_partial(logits, temperatures, seed, self.vocab_start_idx, self.num_embeddings, val, idx)
        vals = torch.empty(self.tp_size, B, dtype=torch.float32, device=logits.device)
        idxs = torch.empty(self.tp_size, B, dtype=torch.int64, device=logits.device)
        dist.all_gather_into_tensor(vals, val)
        dist.all_gather_into_tensor(idxs, idx)
        return K.sample_combine(vals, idxs, out)
