"""SiluAndMul (drop-in for kavor/layers/activation.py): silu(x[:, :I]) * x[:, I:] in one kernel."""
from __future__ import annotations

import torch
from torch import nn

from kavor_b200 import _kernels as K


class SiluAndMul(nn.Module):

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return K.silu_mul(x)
