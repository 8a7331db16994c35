"""Per-kernel CPU restatements of the reference hot path (test infrastructure).

Floating-point ops compute in fp32 torch on the CPU and round to bf16 exactly
where the reference rounds; index work (KV write) is plain integer indexing.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


# ------------------------------------------------------------------ norms
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """layernorm.py:8-39 (eager form :246-251): bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)."""
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    y = (xf * rstd).to(x.dtype)
    return (y.float() * weight.float()).to(x.dtype)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    """layernorm.py:114-140 (eager form :283-288). Returns (out, new_residual);
    the norm uses the fp32 sum, the residual is its bf16 rounding."""
    s = x.float() + residual.float()
    new_residual = s.to(x.dtype)
    rstd = torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    y = (s * rstd).to(x.dtype)
    return (y.float() * weight.float()).to(x.dtype), new_residual


# ------------------------------------------------------------------ RoPE
def cos_sin_cache(head_dim: int, max_position: int, base: float) -> torch.Tensor:
    """rotary_embedding.py:96-102: fp32 [max_position, 1, head_dim] = [cos | sin]."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    freqs = torch.outer(torch.arange(max_position, dtype=torch.float), inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze(1)


def rope(x: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor, interleaved: bool = False) -> torch.Tensor:
    """rotary_embedding.py:56-79 applied with cache[positions] (the pairing of
    test_fused_kernels.py:84-88): rotate pairs (i, i + d/2) — or (2i, 2i+1) when
    interleaved — by theta_i in fp32, round to the input dtype."""
    cs = cache[positions.long()].float()  # [T, 1, d]
    half = x.shape[-1] // 2
    cos, sin = cs[..., :half], cs[..., half:]
    xf = x.float()
    if interleaved:
        x1, x2 = xf[..., 0::2], xf[..., 1::2]
        return torch.stack((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).flatten(-2).to(x.dtype)
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


# ------------------------------------------------------------------ activation / linear / embedding
def silu_mul(x: torch.Tensor) -> torch.Tensor:
    """activation.py:8-11 as the compiled kernel evaluates it: fp32 silu(g) * u, one rounding."""
    g, u = x.float().chunk(2, dim=-1)
    return (F.silu(g) * u).to(x.dtype)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """F.linear with fp32 accumulation, bf16 result (linear.py:50,73,157)."""
    y = x.float() @ weight.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype)


def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int = 0, vocab_end: int | None = None):
    """embed_head.py:34-42 for one shard: rows outside [start, end) are zero."""
    vocab_end = weight.shape[0] + vocab_start if vocab_end is None else vocab_end
    mask = (ids >= vocab_start) & (ids < vocab_end)
    rows = weight[(ids - vocab_start).clamp(0, weight.shape[0] - 1)]
    return rows * mask.unsqueeze(-1).to(rows.dtype)


# ------------------------------------------------------------------ KV cache
def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """flash_attention_kvcache.py:23-34: block = slot // block_size, row = slot % block_size; -1 skipped."""
    bs = k_cache.shape[1]
    for t, slot in enumerate(slot_mapping.tolist()):
        if slot == -1:
            continue
        blk, off = divmod(slot, bs)
        k_cache[blk, off] = key[t]
        v_cache[blk, off] = value[t]


def _gather_kv(cache: torch.Tensor, table: list[int], n: int) -> torch.Tensor:
    bs = cache.shape[1]
    nblk = (n + bs - 1) // bs
    return cache[torch.tensor(table[:nblk], dtype=torch.long)].reshape(-1, *cache.shape[2:])[:n]


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, q_pos0: int) -> torch.Tensor:
    """q [Lq, Hq, d], k/v [Lk, Hkv, d]; query i sees keys j <= q_pos0 + i; fp32 softmax."""
    Lq, Hq, _ = q.shape
    Lk, Hkv, _ = k.shape
    g = Hq // Hkv
    kf = k.float().repeat_interleave(g, dim=1)  # query head h reads kv head h // g
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kf) * scale
    qi = torch.arange(Lq).unsqueeze(1) + q_pos0
    kj = torch.arange(Lk).unsqueeze(0)
    s = s.masked_fill((kj > qi).unsqueeze(0), float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.einsum("hqk,khd->qhd", p, vf)


def paged_decode_attention(q, k_cache, v_cache, block_tables, context_lens, scale) -> torch.Tensor:
    """flash_attn_with_kvcache(q[:,None], k_cache, v_cache, cache_seqlens=context_lens,
    block_table, causal=True) as called at flash_attention_kvcache.py:81-83."""
    B, Hq, d = q.shape
    out = torch.zeros(B, Hq, d, dtype=torch.float32)
    for b in range(B):
        n = int(context_lens[b])
        if n <= 0:
            continue
        table = block_tables[b].tolist()
        k = _gather_kv(k_cache, table, n)
        v = _gather_kv(v_cache, table, n)
        out[b] = _attend(q[b:b + 1], k, v, scale, n - 1)[0]
    return out.to(q.dtype)


def varlen_prefill_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, scale, block_tables=None) -> torch.Tensor:
    """flash_attn_varlen_func(..., causal=True, block_table) as called at
    flash_attention_kvcache.py:76-79; with block_tables, k/v are the paged caches."""
    T, Hq, d = q.shape
    out = torch.zeros(T, Hq, d, dtype=torch.float32)
    cq, ck = cu_seqlens_q.tolist(), cu_seqlens_k.tolist()
    for b in range(len(cq) - 1):
        lq, lk = cq[b + 1] - cq[b], ck[b + 1] - ck[b]
        if lq == 0:
            continue
        if block_tables is not None:
            table = block_tables[b].tolist()
            kb, vb = _gather_kv(k, table, lk), _gather_kv(v, table, lk)
        else:
            kb, vb = k[ck[b]:ck[b + 1]], v[ck[b]:ck[b + 1]]
        out[cq[b]:cq[b + 1]] = _attend(q[cq[b]:cq[b + 1]], kb, vb, scale, lk - lq)
    return out.to(q.dtype)


# ------------------------------------------------------------------ sampler
def greedy(logits: torch.Tensor) -> torch.Tensor:
    """sampler.py:34-44 with T == 0: argmax over fp32 logits, lowest index on ties."""
    return logits.float().argmax(dim=-1)


_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85


def philox4x32_10(ctr: np.ndarray, key0: int) -> np.ndarray:
    """Philox4x32-10 (Salmon et al., SC'11) on counters (c0, c1, 0, 0), key (key0, 0).
    ctr: uint64 array of 64-bit counters; returns uint32 [n, 4]."""
    ctr = np.asarray(ctr, dtype=np.uint64)
    c = [(ctr & 0xFFFFFFFF).astype(np.uint64), (ctr >> np.uint64(32)).astype(np.uint64),
         np.zeros_like(ctr), np.zeros_like(ctr)]
    k0, k1 = np.uint64(key0 & 0xFFFFFFFF), np.uint64(0)
    mask = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = np.uint64(_M0) * c[0]
        p1 = np.uint64(_M1) * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c = [(hi1 ^ c[1] ^ k0) & mask, lo1, (hi0 ^ c[3] ^ k1) & mask, lo0]
        k0 = (k0 + np.uint64(_W0)) & mask
        k1 = (k1 + np.uint64(_W1)) & mask
    return np.stack(c, axis=-1).astype(np.uint32)


def gumbel_scores(logits: torch.Tensor, temperatures: torch.Tensor, seed: int) -> torch.Tensor:
    """Scores of the sampler kernel: logit / T + (-log(-log(u))) with u from
    Philox keyed by seed at counter (b * V + v) / 4, lane (b * V + v) % 4."""
    B, V = logits.shape
    n = np.arange(B * V, dtype=np.uint64)
    r = philox4x32_10(n >> np.uint64(2), seed)[np.arange(B * V), (n & np.uint64(3)).astype(np.int64)]
    u = ((r >> 9).astype(np.float64) + 0.5) / 8388608.0
    g = torch.from_numpy(-np.log(-np.log(u))).view(B, V)
    t = temperatures.double().unsqueeze(1)
    return logits.double() / t + g


def sample(logits: torch.Tensor, temperatures: torch.Tensor, seed: int) -> torch.Tensor:
    scores = gumbel_scores(logits, temperatures.clamp_min(1e-30), seed)
    greedy_rows = temperatures == 0
    out = scores.argmax(dim=-1)
    out[greedy_rows] = greedy(logits[greedy_rows])
    return out
