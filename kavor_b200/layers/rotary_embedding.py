"""Rotary position embedding (drop-in for kavor/layers/rotary_embedding.py).

The fp32 table ``cos_sin_cache`` [max_position, 1, head_size] = [cos | sin] of
``t * inv_freq`` with ``inv_freq = 1 / base**(2j / rotary_dim)`` is built with
the same torch expressions as rotary_embedding.py:96-102, so it is bit-identical
to the reference's table on the same device. ``forward`` rotates q and k in
place with one kernel launch (neox halves, or adjacent pairs when
``interleaved``).
"""
from __future__ import annotations

from functools import lru_cache

import torch
from torch import nn

from kavor_b200 import _kernels as K


def build_cos_sin_cache(rotary_dim: int, max_position: int, base: float) -> torch.Tensor:
    exponents = torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim
    inv_freq = 1.0 / (base ** exponents)
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)


class RotaryEmbedding(nn.Module):

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float,
                 interleaved: bool = False) -> None:
        super().__init__()
        if rotary_dim != head_size:
            raise ValueError("partial rotary embedding is not supported (rotary_dim must equal head_size)")
        self.head_size = head_size
        self.interleaved = interleaved
        self.register_buffer("cos_sin_cache", build_cos_sin_cache(rotary_dim, max_position_embeddings, base),
                             persistent=False)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        return K.rope(positions, query, key, self.cos_sin_cache, self.interleaved)


@lru_cache(1)
def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float, interleaved: bool = False):
    return RotaryEmbedding(head_size, rotary_dim, max_position, base, interleaved)
