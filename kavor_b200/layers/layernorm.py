"""RMSNorm (drop-in for kavor/layers/layernorm.py:RMSNorm).

``forward(x)`` returns a new tensor (2-D [T, H] or strided 3-D [T, heads, H]);
``forward(x, residual)`` adds into ``residual`` in place and returns
``(out, residual)``. Numerics follow layernorm.py:8-39 / 114-140: fp32 inside,
``out = bf16(bf16(x * rstd) * weight)``, the residual stored as bf16 of the
fp32 sum.
"""
from __future__ import annotations

import torch
from torch import nn

from kavor_b200 import _kernels as K


class RMSNorm(nn.Module):

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def rms_forward(self, x: torch.Tensor) -> torch.Tensor:
        return K.rmsnorm(x, self.weight, self.eps)

    def add_rms_forward(self, x: torch.Tensor, residual: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return K.add_rmsnorm(x, residual, self.weight, self.eps)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return self.rms_forward(x)
        return self.add_rms_forward(x, residual)
