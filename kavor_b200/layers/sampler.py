"""Sampler (drop-in for kavor/layers/sampler.py).

Gumbel-max sampling ``argmax(logits / T + Gumbel)`` in one streaming pass per
row, greedy argmax (lowest index on ties) when ``T == 0``. The seed is a
persistent device int32 advanced by one on every call before sampling
(sampler.py:54-59), so a captured CUDA graph advances it on every replay.
"""
from __future__ import annotations

import torch
from torch import nn

from kavor_b200 import _kernels as K


class Sampler(nn.Module):

    def __init__(self):
        super().__init__()
        self.register_buffer("seed", torch.zeros((), dtype=torch.int32, device="cuda"))

    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor, out: torch.Tensor | None = None):
        assert logits.is_contiguous() and temperatures.is_contiguous()
        self.seed.add_(1)
        return K.sample(logits, temperatures, self.seed, out=out)
