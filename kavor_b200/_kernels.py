"""Torch-facing wrappers of the C ABI (one function per entry point).

Each wrapper checks dtypes, devices and layouts the way the reference layers
assert them, passes raw pointers, element strides and torch's current CUDA
stream, and raises ``RuntimeError`` on any failure. Nothing here computes on
the CPU: every op is a launch of a kernel in ``libkavor_b200.so``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_BF16 = torch.bfloat16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _req(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _cuda(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> None:
    _req(isinstance(t, torch.Tensor) and t.is_cuda, f"{name} must be a CUDA tensor")
    if dtype is not None:
        _req(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")


# ------------------------------------------------------------------ workspace
class _Workspace:
    """Per-device scratch buffer for kernels that need one (split-KV decode).

    Grown only outside CUDA-graph capture; superseded buffers are kept alive so
    graphs captured against them stay valid.
    """

    def __init__(self) -> None:
        self.buf: dict[int, torch.Tensor] = {}
        self.retired: list[torch.Tensor] = []

    def reserve(self, nbytes: int, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        cur = self.buf.get(idx)
        if cur is not None and cur.numel() >= nbytes:
            return cur
        _req(not torch.cuda.is_current_stream_capturing(),
             f"decode workspace of {nbytes} bytes must be reserved before CUDA-graph capture")
        if cur is not None:
            self.retired.append(cur)
        new = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        self.buf[idx] = new
        return new


WORKSPACE = _Workspace()


class _ZeroedWorkspace(_Workspace):
    """Per-device workspace of the stream-K GEMM: zero when allocated (its
    hand-off flags must start at zero; every normal launch leaves them zero
    again). One per device, used by launches that are ordered on one stream."""

    def reserve(self, nbytes: int, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        cur = self.buf.get(idx)
        if cur is not None and cur.numel() >= nbytes:
            return cur
        _req(not torch.cuda.is_current_stream_capturing(),
             f"GEMM workspace of {nbytes} bytes must be reserved before CUDA-graph capture")
        if cur is not None:
            self.retired.append(cur)
        new = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        self.buf[idx] = new
        return new

    def reset(self, bits: int = 0) -> None:
        """Zero every workspace again. A hand-off wait that gave up leaves the
        flags it did not consume raised, which a later launch would take for
        fresh partials; so this runs whenever the device error bits are read
        and cleared (the read synchronised the device, and the zeroing is
        finished before the next launch on any stream)."""
        for idx, t in self.buf.items():
            with torch.cuda.device(idx):
                t.zero_()
                torch.cuda.synchronize()


GEMM_WORKSPACE = _ZeroedWorkspace()
_lib.on_cleared_device_error(GEMM_WORKSPACE.reset)


# ------------------------------------------------------------------ KV cache
def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """flash_attention_kvcache.py:37-46 (same layout asserts)."""
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    _req(key.stride(-1) == 1 and value.stride(-1) == 1, "key/value last dim must be contiguous")
    _req(key.stride(1) == head_dim and value.stride(1) == head_dim, "key/value heads must be packed")
    _req(k_cache.stride(1) == D and v_cache.stride(1) == D, "cache rows must hold num_kv_heads*head_dim")
    _req(slot_mapping.numel() == N, "slot_mapping must have one entry per token")
    for t, n in ((key, "key"), (value, "value"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _cuda(t, n, _BF16)
    _cuda(slot_mapping, "slot_mapping", torch.int32)
    _lib.call("kvb_store_kv", key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
              k_cache.data_ptr(), v_cache.data_ptr(), k_cache.size(0), k_cache.stride(0), k_cache.size(1),
              num_heads, head_dim, slot_mapping.data_ptr(), N, _stream())


# ------------------------------------------------------------------ norms
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """layernorm.py:235-258: 2-D [T, H] or 3-D strided [T, heads, H] input, new output tensor."""
    _cuda(x, "x", _BF16)
    _cuda(weight, "weight", _BF16)
    _req(x.stride(-1) == 1, "rmsnorm: last dim must be contiguous")
    n_cols = x.shape[-1]
    _req(weight.numel() == n_cols, "rmsnorm: weight size mismatch")
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if x.dim() == 3:
        tokens, heads = x.shape[0], x.shape[1]
        xs = (x.stride(0), x.stride(1))
        os_ = (out.stride(0), out.stride(1))
    else:
        _req(x.dim() == 2, "rmsnorm: 2-D or 3-D input")
        tokens, heads = x.shape[0], 1
        xs = (x.stride(0), 0)
        os_ = (out.stride(0), 0)
    _lib.call("kvb_rmsnorm", x.data_ptr(), xs[0], xs[1], out.data_ptr(), os_[0], os_[1], weight.data_ptr(),
              tokens, heads, n_cols, float(eps), _stream())
    return out


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """layernorm.py:260-288: residual updated in place, returns (out, residual)."""
    for t, n in ((x, "x"), (residual, "residual"), (weight, "weight")):
        _cuda(t, n, _BF16)
    _req(x.dim() == 2 and x.is_contiguous() and residual.is_contiguous() and x.shape == residual.shape,
         "add_rmsnorm: contiguous [tokens, hidden] x and residual")
    if out is None:
        out = torch.empty_like(x)
    _lib.call("kvb_add_rmsnorm", x.data_ptr(), residual.data_ptr(), out.data_ptr(), weight.data_ptr(),
              x.shape[0], x.shape[1], float(eps), _stream())
    return out, residual


# ------------------------------------------------------------------ RoPE
def rope(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor, cos_sin: torch.Tensor,
         interleaved: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """rotary_embedding.py:104-120: in place on strided [T, heads, head_dim] views."""
    _cuda(query, "query", _BF16)
    _cuda(key, "key", _BF16)
    _cuda(positions, "positions", torch.int64)
    _cuda(cos_sin, "cos_sin_cache", torch.float32)
    _req(query.stride(-1) == 1 and key.stride(-1) == 1, "rope: last dim must be contiguous")
    _req(cos_sin.is_contiguous(), "rope: cos_sin cache must be contiguous")
    head_dim = query.shape[-1]
    _lib.call("kvb_rope", query.data_ptr(), query.stride(0), query.stride(1), key.data_ptr(), key.stride(0),
              key.stride(1), positions.data_ptr(), cos_sin.data_ptr(), cos_sin.shape[0], query.shape[0],
              query.shape[1], key.shape[1], head_dim, int(interleaved), _stream())
    return query, key


def qknorm_rope_store(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int,
                      q_weight: torch.Tensor | None, k_weight: torch.Tensor | None, eps: float,
                      positions: torch.Tensor, cos_sin: torch.Tensor, interleaved: bool,
                      k_cache: torch.Tensor | None, v_cache: torch.Tensor | None,
                      slot_mapping: torch.Tensor | None) -> None:
    """qwen3.py:80-89 + the KV write of flash_attention_kvcache.py:72, fused, in place on qkv."""
    _cuda(qkv, "qkv", _BF16)
    _cuda(positions, "positions", torch.int64)
    _cuda(cos_sin, "cos_sin_cache", torch.float32)
    _req(qkv.dim() == 2 and qkv.stride(-1) == 1, "qkv must be [tokens, (Hq+2Hkv)*head_dim]")
    apply_norm = q_weight is not None
    has_cache = k_cache is not None and k_cache.numel() > 0
    if has_cache:
        _cuda(slot_mapping, "slot_mapping", torch.int32)
        _req(slot_mapping.numel() == qkv.shape[0], "slot_mapping must have one entry per token")
    _lib.call("kvb_qknorm_rope_store", qkv.data_ptr(), qkv.stride(0), qkv.shape[0], num_q_heads, num_kv_heads,
              head_dim, q_weight.data_ptr() if apply_norm else None, k_weight.data_ptr() if apply_norm else None,
              float(eps), int(apply_norm), positions.data_ptr(), cos_sin.data_ptr(), cos_sin.shape[0],
              int(interleaved), k_cache.data_ptr() if has_cache else None,
              v_cache.data_ptr() if has_cache else None, k_cache.size(0) if has_cache else 0,
              k_cache.stride(0) if has_cache else 0, k_cache.size(1) if has_cache else 0,
              slot_mapping.data_ptr() if has_cache else None, _stream())


# ------------------------------------------------------------------ activation / embedding
def silu_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """activation.py:8-11: silu(x[:, :I]) * x[:, I:]."""
    _cuda(x, "x", _BF16)
    _req(x.dim() == 2 and x.stride(-1) == 1 and x.shape[1] % 2 == 0, "silu_mul: [tokens, 2*I] input")
    inter = x.shape[1] // 2
    if out is None:
        out = torch.empty(x.shape[0], inter, dtype=x.dtype, device=x.device)
    _lib.call("kvb_silu_mul", x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), x.shape[0], inter,
              _stream())
    return out


def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int, vocab_end: int, vocab_size: int,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """embed_head.py:34-42 lookup with the out-of-shard rows zeroed."""
    _cuda(ids, "input_ids", torch.int64)
    _cuda(weight, "weight", _BF16)
    _req(weight.is_contiguous(), "embedding weight must be contiguous")
    ids = ids.reshape(-1)
    if out is None:
        out = torch.empty(ids.numel(), weight.shape[1], dtype=weight.dtype, device=weight.device)
    _lib.call("kvb_embedding", ids.data_ptr(), weight.data_ptr(), out.data_ptr(), ids.numel(), weight.shape[1],
              vocab_start, vocab_end, vocab_size, _stream())
    return out


# ------------------------------------------------------------------ attention
def decode_workspace_bytes(batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int, max_blocks: int,
                           block_size: int, num_splits: int = 0) -> int:
    n = ctypes.c_size_t(0)
    _lib.call("kvb_paged_decode_attn_workspace_size", batch, num_q_heads, num_kv_heads, head_dim, max_blocks,
              block_size, num_splits, ctypes.byref(n))
    return int(n.value)


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float,
                           out: torch.Tensor | None = None, num_splits: int = 0,
                           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """flash_attention_kvcache.py:80-83: q [B, Hq, hd] over the paged cache -> [B, Hq, hd]."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _cuda(t, n, _BF16)
    _cuda(block_tables, "block_tables", torch.int32)
    _cuda(context_lens, "context_lens", torch.int32)
    _req(q.dim() == 3 and q.stride(-1) == 1, "decode q must be [batch, heads, head_dim]")
    _req(block_tables.dim() == 2 and block_tables.stride(1) == 1, "block_tables must be [batch, max_blocks]")
    B, Hq, hd = q.shape
    nblk, bs, Hkv, _ = k_cache.shape
    _req(k_cache.stride(1) == Hkv * hd and k_cache.stride(2) == hd, "k_cache rows must be packed")
    _req(v_cache.stride(0) == k_cache.stride(0), "k/v caches must share the page stride")
    if out is None:
        out = torch.empty(B, Hq, hd, dtype=q.dtype, device=q.device)
    maxb = block_tables.shape[1]
    need = decode_workspace_bytes(B, Hq, Hkv, hd, maxb, bs, num_splits)
    if need and workspace is None:
        workspace = WORKSPACE.reserve(need, q.device)
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
    _lib.call("kvb_paged_decode_attn", q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(),
              v_cache.data_ptr(), nblk, k_cache.stride(0), bs, block_tables.data_ptr(), block_tables.stride(0),
              maxb, context_lens.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), B, Hq, Hkv, hd,
              float(scale), num_splits, ws_ptr, ws_len, _stream())
    return out


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                      cu_seqlens_k: torch.Tensor, max_seqlen_q: int, scale: float,
                      block_tables: torch.Tensor | None = None, out: torch.Tensor | None = None,
                      tensor_cores: bool = True) -> torch.Tensor:
    """flash_attention_kvcache.py:73-79. With block_tables, k/v are the paged caches
    [num_blocks, block_size, Hkv, hd]; otherwise contiguous-row [total_k, Hkv, hd] views.
    tensor_cores=False forces the warp-MMA kernel (the tcgen05 one is the default)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _cuda(t, n, _BF16)
    _cuda(cu_seqlens_q, "cu_seqlens_q", torch.int32)
    _cuda(cu_seqlens_k, "cu_seqlens_k", torch.int32)
    _req(q.dim() == 3 and q.stride(-1) == 1, "prefill q must be [total_q, heads, head_dim]")
    T, Hq, hd = q.shape
    batch = cu_seqlens_q.numel() - 1
    if out is None:
        out = torch.empty(T, Hq, hd, dtype=q.dtype, device=q.device)
    if block_tables is not None:
        _cuda(block_tables, "block_tables", torch.int32)
        nblk, bs, Hkv, _ = k.shape
        _req(v.stride(0) == k.stride(0), "k/v caches must share the page stride")
        _lib.call("kvb_prefill_attn", q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), 0, 0, v.data_ptr(),
                  0, 0, nblk, k.stride(0), bs, block_tables.data_ptr(), block_tables.stride(0),
                  block_tables.shape[1], cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), batch,
                  int(max_seqlen_q), out.data_ptr(), out.stride(0), out.stride(1), Hq, Hkv, hd, float(scale),
                  T if tensor_cores else 0, 0, _stream())
    else:
        Hkv = k.shape[1]
        _req(k.stride(-1) == 1 and v.stride(-1) == 1, "k/v last dim must be contiguous")
        _lib.call("kvb_prefill_attn", q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0),
                  k.stride(1), v.data_ptr(), v.stride(0), v.stride(1), 0, 0, 0, None, 0, 0,
                  cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), batch, int(max_seqlen_q), out.data_ptr(),
                  out.stride(0), out.stride(1), Hq, Hkv, hd, float(scale), T if tensor_cores else 0,
                  k.shape[0] if tensor_cores else 0, _stream())
    return out


# ------------------------------------------------------------------ GEMM
def gemm_workspace_bytes(M: int, N: int, K: int, splits: int = 0) -> int:
    n = ctypes.c_size_t(0)
    _lib.call("kvb_gemm_workspace_size", M, N, K, splits, ctypes.byref(n))
    return int(n.value)


def gemm_plan(M: int, N: int, K: int, splits: int = 0, gated: bool = False) -> dict:
    """Tiling the GEMM picks for this shape (token tile, K splits, units, CTAs)."""
    out = (ctypes.c_int * 4)()
    _lib.call("kvb_gemm_plan", M, N, K, splits, int(gated), out)
    return {"mt": out[0], "splits": out[1], "units": out[2], "grid": out[3]}


def set_pdl(enable: bool) -> None:
    """Programmatic dependent launch for every later kernel launch of this
    process (each kernel is scheduled while the one before it on the stream
    still runs and waits at its start for it; results are unchanged)."""
    _lib.call("kvb_set_pdl", 1 if enable else 0)


def gemm_set_l2_prefetch(ksteps: int) -> None:
    """Weight K-steps the GEMM producer prefetches into L2 ahead of its TMA
    loads, for every later launch in this process (0 = off, the default)."""
    _lib.call("kvb_gemm_set_l2_prefetch", int(ksteps))


def gemm(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """y = x @ weight^T on tcgen05 tensor cores (bf16 in/out, fp32 accumulate)."""
    _cuda(x, "x", _BF16)
    _cuda(weight, "weight", _BF16)
    _req(x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1], "gemm: x [M, K], weight [N, K]")
    _req(x.stride(1) == 1 and weight.stride(1) == 1, "gemm: rows must be contiguous")
    M, K = x.shape
    N = weight.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    # the K split reduces through distributed shared memory: no workspace
    _lib.call("kvb_gemm_bf16", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), out.data_ptr(),
              out.stride(0), M, N, K, splits, None, 0, _stream())
    return out


def gemm_pair_plan(M: int, N: int, K: int, splits: int = 0, gated: bool = False) -> dict:
    """Tiling of the CTA-pair GEMM for this shape (token tile, K splits, tiles, CTAs)."""
    out = (ctypes.c_int * 4)()
    _lib.call("kvb_gemm_pair_plan", M, N, K, splits, int(gated), out)
    return {"mt": out[0], "splits": out[1], "tiles": out[2], "ctas": out[3]}


def gemm_pair(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """y = x @ weight^T on CTA pairs (tcgen05 cta_group::2), bf16 in/out, fp32 accumulate."""
    _cuda(x, "x", _BF16)
    _cuda(weight, "weight", _BF16)
    _req(x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1], "gemm_pair: x [M, K], weight [N, K]")
    _req(x.stride(1) == 1 and weight.stride(1) == 1, "gemm_pair: rows must be contiguous")
    M, K = x.shape
    N = weight.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    _lib.call("kvb_gemm_pair_bf16", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), out.data_ptr(),
              out.stride(0), M, N, K, splits, _stream())
    return out


def gemm_pair_silu(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None,
                   splits: int = 0) -> torch.Tensor:
    """silu(x @ w_gate^T) * (x @ w_up^T) for the merged [gate | up] weight on CTA pairs."""
    _cuda(x, "x", _BF16)
    _cuda(weight, "weight", _BF16)
    _req(x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1] and weight.shape[0] % 2 == 0,
         "gemm_pair_silu: x [M, K], weight [2*I, K]")
    _req(x.stride(1) == 1 and weight.stride(1) == 1, "gemm_pair_silu: rows must be contiguous")
    M, K = x.shape
    inter = weight.shape[0] // 2
    if out is None:
        out = torch.empty(M, inter, dtype=x.dtype, device=x.device)
    _lib.call("kvb_gemm_pair_silu_bf16", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0),
              out.data_ptr(), out.stride(0), M, inter, K, splits, _stream())
    return out


def gemm_sk_plan(M: int, N: int, K: int, gated: bool = False) -> dict:
    """Stream-K GEMM plan for this shape: token tile, tiles, K-steps per tile, pairs."""
    out = (ctypes.c_int * 4)()
    _lib.call("kvb_gemm_sk_plan", M, N, K, int(gated), out)
    return {"mt": out[0], "tiles": out[1], "kb": out[2], "pairs": out[3]}


def gemm_sk_set_plan(mt: int = 0, pairs: int = 0) -> None:
    """Force the stream-K GEMM's token tile and pair count for later launches
    (0 = planned); a tuning knob for sweeps."""
    _lib.call("kvb_gemm_sk_set_plan", int(mt), int(pairs))


def gemm_sk_workspace_bytes(M: int, N: int, K: int, gated: bool = False) -> int:
    n = ctypes.c_size_t(0)
    _lib.call("kvb_gemm_sk_workspace_size", M, N, K, int(gated), ctypes.byref(n))
    return int(n.value)


def _gemm_sk_args(x, weight, name, gated):
    _cuda(x, "x", _BF16)
    _cuda(weight, "weight", _BF16)
    _req(x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1], f"{name}: x [M, K], weight [N, K]")
    _req(x.stride(1) == 1 and weight.stride(1) == 1, f"{name}: rows must be contiguous")
    if gated:
        _req(weight.shape[0] % 2 == 0, f"{name}: weight [2*I, K]")
    M, K = x.shape
    N = weight.shape[0] // 2 if gated else weight.shape[0]
    ws = GEMM_WORKSPACE.reserve(max(gemm_sk_workspace_bytes(M, N, K, gated), _gemm_sk_workspace_max()), x.device)
    return M, N, K, ws


_SK_WS_MAX: int | None = None


def _gemm_sk_workspace_max() -> int:
    """The largest workspace any plan needs on this device (every pair, 256-token
    tiles), reserved at the first call so that no later shape grows it (nor has
    to during CUDA-graph capture)."""
    global _SK_WS_MAX
    if _SK_WS_MAX is None:
        _SK_WS_MAX = gemm_sk_workspace_bytes(256, 1 << 20, 1 << 16)
    return _SK_WS_MAX


def gemm_sk(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ weight^T on CTA pairs with the stream-K schedule (bf16 in/out, fp32 accumulate)."""
    M, N, K, ws = _gemm_sk_args(x, weight, "gemm_sk", False)
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    _lib.call("kvb_gemm_sk_bf16", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), out.data_ptr(),
              out.stride(0), M, N, K, ws.data_ptr(), ws.numel(), _stream())
    return out


def gemm_sk_silu(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(x @ w_gate^T) * (x @ w_up^T) for the merged [gate | up] weight, stream-K CTA pairs."""
    M, inter, K, ws = _gemm_sk_args(x, weight, "gemm_sk_silu", True)
    if out is None:
        out = torch.empty(M, inter, dtype=x.dtype, device=x.device)
    _lib.call("kvb_gemm_sk_silu_bf16", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0),
              out.data_ptr(), out.stride(0), M, inter, K, ws.data_ptr(), ws.numel(), _stream())
    return out


def gemm_silu(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None,
              splits: int = 0) -> torch.Tensor:
    """silu(x @ w_gate^T) * (x @ w_up^T) for the merged [gate | up] weight, one kernel."""
    _cuda(x, "x", _BF16)
    _cuda(weight, "weight", _BF16)
    _req(x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1] and weight.shape[0] % 2 == 0,
         "gemm_silu: x [M, K], weight [2*I, K]")
    _req(x.stride(1) == 1 and weight.stride(1) == 1, "gemm_silu: rows must be contiguous")
    M, K = x.shape
    inter = weight.shape[0] // 2
    if out is None:
        out = torch.empty(M, inter, dtype=x.dtype, device=x.device)
    _lib.call("kvb_gemm_silu_bf16", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), out.data_ptr(),
              out.stride(0), M, inter, K, splits, None, 0, _stream())
    return out


# ------------------------------------------------------------------ sampler
def sample(logits: torch.Tensor, temperatures: torch.Tensor, seed: torch.Tensor,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """sampler.py:56-66 (seed is read, not advanced)."""
    _cuda(logits, "logits", _BF16)
    _cuda(temperatures, "temperatures", torch.float32)
    _cuda(seed, "seed", torch.int32)
    _req(logits.dim() == 2 and logits.stride(-1) == 1 and temperatures.is_contiguous(), "sampler layouts")
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    _lib.call("kvb_sample", logits.data_ptr(), logits.stride(0), temperatures.data_ptr(), seed.data_ptr(),
              out.data_ptr(), logits.shape[0], logits.shape[1], _stream())
    return out


def sample_partial(logits: torch.Tensor, temperatures: torch.Tensor, seed: torch.Tensor, vocab_offset: int,
                   vocab_total: int, best_val: torch.Tensor, best_idx: torch.Tensor) -> None:
    _cuda(logits, "logits", _BF16)
    _req(logits.dim() == 2 and logits.stride(-1) == 1, "sampler layouts")
    _lib.call("kvb_sample_partial", logits.data_ptr(), logits.stride(0), temperatures.data_ptr(), seed.data_ptr(),
              best_val.data_ptr(), best_idx.data_ptr(), logits.shape[0], logits.shape[1], vocab_offset,
              vocab_total, _stream())


def sample_combine(vals: torch.Tensor, idxs: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    world, batch = vals.shape
    _lib.call("kvb_sample_combine", vals.data_ptr(), idxs.data_ptr(), world, out.data_ptr(), batch, _stream())
    return out
