"""Tensor-parallel linear layers (drop-in for kavor/layers/linear.py).

Sharding and checkpoint loaders follow linear.py:8-160: column-parallel layers
split the output rows across ranks (QKV rows ordered [q | k | v] per rank,
gate/up rows [gate | up] per rank), row-parallel layers split the input
columns and all-reduce the partial products (bias added on rank 0 only).
All projections go through ``linear()``, the single GEMM entry point of the
package, and the MLP's gate-up projection + SiluAndMul through
``gate_up_silu()``. Which GEMM runs is a process-wide choice
(``set_gemm_backend``): "auto" (the default: the package's stream-K kernel
for decode batches on the weights where it measured faster than cuBLAS on the
B200 — the full-vocabulary LM head — and torch's F.linear for the rest),
"cublas" (torch's F.linear, the reference's own GEMM, everywhere), "tcgen05"
(this package's kernels everywhere: up to SK_MAX_TOKENS tokens
the stream-K CTA-pair kernel kvb_gemm_sk_bf16 / kvb_gemm_sk_silu_bf16, above
it the persistent single-CTA kernel kvb_gemm_bf16 / kvb_gemm_silu_bf16) or
"tcgen05_pair" (the cluster-split CTA-pair kernel, kvb_gemm_pair_bf16, and
its fused form kvb_gemm_pair_silu_bf16).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn


def divide(numerator: int, denominator: int) -> int:
    if numerator % denominator:
        raise ValueError(f"{numerator} is not divisible by {denominator}")
    return numerator // denominator


GEMM_BACKENDS = ("auto", "cublas", "tcgen05", "tcgen05_pair")
_GEMM_BACKEND = "auto"


def set_gemm_backend(name: str) -> None:
    global _GEMM_BACKEND
    if name not in GEMM_BACKENDS:
        raise ValueError(f"unknown GEMM backend {name!r} (one of {GEMM_BACKENDS})")
    _GEMM_BACKEND = name


def gemm_backend() -> str:
    return _GEMM_BACKEND


# Token counts at or below which the "tcgen05" backend runs the stream-K
# CTA-pair kernel (decode batches); above, the persistent single-CTA kernel.
SK_MAX_TOKENS = 256
# "auto": weights of at least this many elements run on the stream-K kernel at
# decode batches. Measured on one B200 (graph-timed, weights streamed from HBM):
# the Qwen3-8B LM head [151936, 4096] takes 183-257 us against cuBLAS's
# 195-283 us from 1 to 256 tokens; every projection of a decoder layer and the
# vocabulary shard at TP=8 ([18992, 4096]) is faster on cuBLAS.
SK_AUTO_MIN_WEIGHT = 500_000_000


def auto_uses_stream_k(M: int, N: int, K: int) -> bool:
    """Whether the "auto" backend runs y[M, N] = x[M, K] W[N, K]^T on the
    stream-K kernel (else F.linear)."""
    return M <= SK_MAX_TOKENS and N * K >= SK_AUTO_MIN_WEIGHT and K % 64 == 0


def _use_sk(x: torch.Tensor, weight: torch.Tensor) -> bool:
    return x.is_cuda and auto_uses_stream_k(x.shape[0], weight.shape[0], weight.shape[1])


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x W^T (+ b) in bf16 with fp32 accumulation."""
    if _GEMM_BACKEND == "auto" and _use_sk(x, weight):
        from kavor_b200 import _kernels as K

        y = K.gemm_sk(x, weight, out=out)
        if bias is not None:
            y.add_(bias)
        return y
    if _GEMM_BACKEND not in ("cublas", "auto"):
        from kavor_b200 import _kernels as K

        if _GEMM_BACKEND == "tcgen05":
            fn = K.gemm_sk if x.shape[0] <= SK_MAX_TOKENS and x.shape[1] % 64 == 0 else K.gemm
        else:
            fn = K.gemm_pair
        y = fn(x, weight, out=out)
        if bias is not None:
            y.add_(bias)
        return y
    if out is None:
        return F.linear(x, weight, bias)
    torch.matmul(x, weight.t(), out=out)
    if bias is not None:
        out.add_(bias)
    return out


def gate_up_silu(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor | None:
    """silu(x W_gate^T) * (x W_up^T) for the merged [gate | up] weight in one
    kernel of the active backend (the reference's rounding points); None when
    the backend has no fused form (cuBLAS: the caller runs the projection and
    SiluAndMul)."""
    if _GEMM_BACKEND in ("cublas", "auto"):  # auto: no gate-up shape is faster fused (see SK_AUTO_MIN_WEIGHT)
        return None
    from kavor_b200 import _kernels as K

    if _GEMM_BACKEND == "tcgen05":
        return (K.gemm_sk_silu if x.shape[0] <= SK_MAX_TOKENS and x.shape[1] % 64 == 0 else K.gemm_silu)(x, weight)
    return K.gemm_pair_silu(x, weight)


def _tp() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


class LinearBase(nn.Module):

    def __init__(self, input_size: int, output_size: int, bias: bool = False, tp_dim: int | None = None):
        super().__init__()
        self.tp_dim = tp_dim
        self.tp_rank, self.tp_size = _tp()
        self.weight = nn.Parameter(torch.empty(output_size, input_size))
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size))
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, *args):
        raise NotImplementedError

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class ReplicatedLinear(LinearBase):

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__(input_size, output_size, bias)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param.data.copy_(loaded_weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return linear(x, self.weight, self.bias)


class ColumnParallelLinear(LinearBase):

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        _, tp_size = _tp()
        super().__init__(input_size, divide(output_size, tp_size), bias, 0)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        shard = param.data.size(self.tp_dim)
        param.data.copy_(loaded_weight.narrow(self.tp_dim, self.tp_rank * shard, shard))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return linear(x, self.weight, self.bias)


class MergedColumnParallelLinear(ColumnParallelLinear):

    def __init__(self, input_size: int, output_sizes: list[int], bias: bool = False):
        self.output_sizes = output_sizes
        super().__init__(input_size, sum(output_sizes), bias)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: int):
        offset = sum(self.output_sizes[:loaded_shard_id]) // self.tp_size
        size = self.output_sizes[loaded_shard_id] // self.tp_size
        dst = param.data.narrow(self.tp_dim, offset, size)
        dst.copy_(loaded_weight.chunk(self.tp_size, self.tp_dim)[self.tp_rank])


class QKVParallelLinear(ColumnParallelLinear):

    def __init__(self, output_size: int, hidden_size: int, head_size: int, total_num_heads: int,
                 total_num_kv_heads: int | None = None, q_gate: bool = False, bias: bool = False):
        _, tp_size = _tp()
        self.q_mult = 2 if q_gate else 1
        total_num_kv_heads = total_num_kv_heads or total_num_heads
        self.head_size = head_size
        self.num_heads = divide(total_num_heads, tp_size)
        self.num_kv_heads = divide(total_num_kv_heads, tp_size)
        super().__init__(hidden_size, output_size, bias)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: str):
        if loaded_shard_id not in ("q", "k", "v"):
            raise ValueError(f"unknown qkv shard {loaded_shard_id!r}")
        q_size = self.q_mult * self.num_heads * self.head_size
        kv_size = self.num_kv_heads * self.head_size
        offset, size = {"q": (0, q_size), "k": (q_size, kv_size), "v": (q_size + kv_size, kv_size)}[loaded_shard_id]
        dst = param.data.narrow(self.tp_dim, offset, size)
        dst.copy_(loaded_weight.chunk(self.tp_size, self.tp_dim)[self.tp_rank])


class RowParallelLinear(LinearBase):

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        _, tp_size = _tp()
        super().__init__(divide(input_size, tp_size), output_size, bias, 1)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        if param.data.ndim == 1:
            param.data.copy_(loaded_weight)
            return
        shard = param.data.size(self.tp_dim)
        param.data.copy_(loaded_weight.narrow(self.tp_dim, self.tp_rank * shard, shard))

    def forward(self, x: torch.Tensor, reduce: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
        """``reduce=False`` returns the rank-local partial sum (written into
        ``out`` when given) so the caller can fuse the all-reduce with what follows."""
        y = linear(x, self.weight, self.bias if self.tp_rank == 0 else None, out=out)
        if reduce and self.tp_size > 1:
            dist.all_reduce(y)
        return y
