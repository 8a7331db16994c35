"""Kernel parity: every sm_100a kernel of libkavor_b200.so against the CPU oracle
on seeded inputs. Integer/byte work (KV write, embedding, residual, greedy
argmax) must be bit-exact; floating-point outputs use the reference suite's
tolerances (tests/test_fused_kernels.py there: 2e-2) or the per-layer
parity bound (max-abs 2e-2, rel 1e-2)."""
import pytest
import torch

import cases
from oracle import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"
EPS = 1e-6


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from kavor_b200 import _lib as L

    L.load()
    L.device_error(clear=True)
    yield
    assert L.device_error(clear=True) == 0, "a kernel raised a device-side error bit"


def K():
    from kavor_b200 import _kernels

    return _kernels


def close(a, b, atol=2e-2, rtol=1e-2):
    torch.testing.assert_close(a.float().cpu(), b.float().cpu(), atol=atol, rtol=rtol)


def g(seed):
    return torch.Generator().manual_seed(seed)


# ------------------------------------------------------------------ KV write
def test_store_kvcache_bit_exact_with_padding_slots():
    T, Hq, Hkv, hd, bs, nblk = 37, 8, 4, 128, 256, 6
    qkv = torch.randn(T, (Hq + 2 * Hkv) * hd, generator=g(0)).to(torch.bfloat16)
    k = qkv[:, Hq * hd:(Hq + Hkv) * hd].view(T, Hkv, hd)
    v = qkv[:, (Hq + Hkv) * hd:].view(T, Hkv, hd)
    slots = torch.randperm(nblk * bs, generator=g(1))[:T].to(torch.int32)
    slots[::5] = -1
    pool = torch.randn(nblk, 2, bs, Hkv, hd, generator=g(2)).to(torch.bfloat16)
    ref = pool.clone()
    ops.store_kvcache(k, v, ref[:, 0], ref[:, 1], slots)
    dpool = pool.to(DEV)
    dqkv = qkv.to(DEV)
    K().store_kvcache(dqkv[:, Hq * hd:(Hq + Hkv) * hd].view(T, Hkv, hd), dqkv[:, (Hq + Hkv) * hd:].view(T, Hkv, hd),
                      dpool[:, 0], dpool[:, 1], slots.to(DEV))
    assert torch.equal(dpool.cpu(), ref)


# ------------------------------------------------------------------ norms
@pytest.mark.parametrize("shape,view", [((128, 4096), False), ((1, 4096), False), ((7, 1024), False),
                                        ((3, 5120), False), ((37, 32, 128), True), ((5, 8, 80), True)])
def test_rmsnorm_matches_oracle(shape, view):
    w = (torch.randn(shape[-1], generator=g(3)) * 0.1 + 1).to(torch.bfloat16)
    if view:
        buf = torch.randn(shape[0], shape[1] * 3, shape[2], generator=g(4)).to(torch.bfloat16)
        x = buf[:, :shape[1], :]
        dx = buf.to(DEV)[:, :shape[1], :]
    else:
        x = torch.randn(shape, generator=g(4)).to(torch.bfloat16)
        dx = x.to(DEV)
    ref = ops.rmsnorm(x, w, EPS)
    out = K().rmsnorm(dx, w.to(DEV), EPS)
    close(out, ref, 2e-2, 2e-2)
    assert (out.cpu() == ref).float().mean() > 0.98  # same rounding points: almost all bit-equal


def test_add_rmsnorm_residual_bit_exact():
    w = (torch.randn(4096, generator=g(5)) * 0.1 + 1).to(torch.bfloat16)
    x = torch.randn(256, 4096, generator=g(6)).to(torch.bfloat16)
    r = torch.randn(256, 4096, generator=g(7)).to(torch.bfloat16)
    ref_out, ref_res = ops.add_rmsnorm(x, r, w, EPS)
    dr = r.to(DEV)
    out, res = K().add_rmsnorm(x.to(DEV), dr, w.to(DEV), EPS)
    assert res.data_ptr() == dr.data_ptr()  # in place, like layernorm.py:280
    assert torch.equal(res.cpu(), ref_res)
    close(out, ref_out, 2e-2, 2e-2)


# ------------------------------------------------------------------ RoPE
@pytest.mark.parametrize("interleaved", [False, True])
def test_rope_matches_oracle(interleaved):
    from kavor_b200.layers.rotary_embedding import build_cos_sin_cache

    T, Hq, Hkv, hd, max_pos = 64, 32, 8, 128, 4096
    cache = build_cos_sin_cache(hd, max_pos, 1e6)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * hd, generator=g(8)).to(torch.bfloat16)
    pos = torch.randint(0, max_pos, (T,), generator=g(9))
    q = qkv[:, :Hq * hd].view(T, Hq, hd)
    k = qkv[:, Hq * hd:(Hq + Hkv) * hd].view(T, Hkv, hd)
    q_ref, k_ref = ops.rope(q, pos, cache, interleaved), ops.rope(k, pos, cache, interleaved)
    d = qkv.to(DEV)
    dq = d[:, :Hq * hd].view(T, Hq, hd)
    dk = d[:, Hq * hd:(Hq + Hkv) * hd].view(T, Hkv, hd)
    K().rope(pos.to(DEV), dq, dk, cache.to(DEV).contiguous(), interleaved)
    close(dq, q_ref, 2e-2, 2e-2)
    close(dk, k_ref, 2e-2, 2e-2)


@pytest.mark.parametrize("hq,hkv,qk_norm,interleaved", [
    (16, 8, True, False), (32, 8, True, False), (4, 1, True, False), (64, 8, True, False),
    (32, 8, False, False),   # Mistral: no q/k norm
    (16, 2, False, True),    # ERNIE 4.5: no q/k norm, interleaved pairs
])
def test_fused_qknorm_rope_store(hq, hkv, qk_norm, interleaved):
    from kavor_b200.layers.rotary_embedding import build_cos_sin_cache

    T, hd, bs, nblk = 19, 128, 256, 3
    cache = build_cos_sin_cache(hd, 40960, 1e6)
    qkv = torch.randn(T, (hq + 2 * hkv) * hd, generator=g(10)).to(torch.bfloat16)
    qw = (torch.randn(hd, generator=g(11)) * 0.1 + 1).to(torch.bfloat16)
    kw = (torch.randn(hd, generator=g(12)) * 0.1 + 1).to(torch.bfloat16)
    pos = torch.randint(0, 40960, (T,), generator=g(13))
    slots = torch.randperm(nblk * bs, generator=g(14))[:T].to(torch.int32)
    slots[3] = -1
    q = qkv[:, :hq * hd].view(T, hq, hd)
    k = qkv[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd)
    v = qkv[:, (hq + hkv) * hd:].view(T, hkv, hd)
    qn, kn = (ops.rmsnorm(q, qw, EPS), ops.rmsnorm(k, kw, EPS)) if qk_norm else (q, k)
    q_ref = ops.rope(qn, pos, cache, interleaved)
    k_ref = ops.rope(kn, pos, cache, interleaved)
    pool = torch.zeros(nblk, 2, bs, hkv, hd, dtype=torch.bfloat16, device=DEV)
    d = qkv.to(DEV)
    K().qknorm_rope_store(d, hq, hkv, hd, qw.to(DEV) if qk_norm else None, kw.to(DEV) if qk_norm else None, EPS,
                          pos.to(DEV), cache.to(DEV).contiguous(), interleaved, pool[:, 0], pool[:, 1], slots.to(DEV))
    dq = d[:, :hq * hd].view(T, hq, hd).cpu()
    dk = d[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd).cpu()
    close(dq, q_ref, 2e-2, 2e-2)
    close(dk, k_ref, 2e-2, 2e-2)
    # the cache holds exactly the kernel's own k and the untouched v
    ref_pool = torch.zeros(nblk, 2, bs, hkv, hd, dtype=torch.bfloat16)
    ops.store_kvcache(dk, v, ref_pool[:, 0], ref_pool[:, 1], slots)
    assert torch.equal(pool.cpu(), ref_pool)


# ------------------------------------------------------------------ activation / embedding
def test_silu_mul_matches_oracle():
    x = (torch.randn(33, 2 * 3072, generator=g(15)) * 3).to(torch.bfloat16)
    close(K().silu_mul(x.to(DEV)), ops.silu_mul(x), atol=1e-5, rtol=2 ** -7)


def test_embedding_shard_is_exact():
    V, H = 1000, 512
    w = torch.randn(V, H, generator=g(16)).to(torch.bfloat16)
    ids = torch.randint(0, 4 * V, (77,), generator=g(17))
    start = 2 * V
    out = K().embedding(ids.to(DEV), w.to(DEV), start, start + V, 4 * V)
    assert torch.equal(out.cpu(), ops.embedding(ids, w, start, start + V))


# ------------------------------------------------------------------ decode attention
def _decode_case(B, hq, hkv, ctx, seed, nan_tail=False):
    bs = 256
    need = [max(1, (c + bs - 1) // bs) for c in ctx]
    nblk = sum(need) + 2
    perm = torch.randperm(nblk, generator=g(seed)).tolist()
    width = max(need)
    tables, k = [], 0
    for n in need:
        tables.append(perm[k:k + n] + [-1] * (width - n))
        k += n
    pool = torch.randn(nblk, 2, bs, hkv, 128, generator=g(seed + 1)).to(torch.bfloat16)
    if nan_tail:  # stale bytes after each context must not leak into the result
        for b, c in enumerate(ctx):
            for j, blk in enumerate(tables[b][:need[b]]):
                lo = max(0, c - j * bs)
                if lo < bs:
                    pool[blk, :, lo:] = float("nan")
    q = torch.randn(B, hq, 128, generator=g(seed + 2)).to(torch.bfloat16)
    return q, pool, torch.tensor(tables, dtype=torch.int32), torch.tensor(ctx, dtype=torch.int32)


@pytest.mark.parametrize("B,hq,hkv,ctx,splits", [
    (16, 16, 8, None, 0),                    # the one-layer case batch (0.6B heads, ctx U[100,1024])
    (4, 32, 8, [1, 63, 64, 65], 0),          # tile-boundary contexts
    (3, 4, 1, [1024, 1000, 257], 0),         # TP8-like: 1 kv head, group 4
    (2, 64, 8, [700, 1500], 0),              # group 8 (Qwen3-32B TP1)
    (5, 32, 8, [1024, 900, 0, 300, 1025], 1),  # a padding row (ctx 0), one split
    (5, 32, 8, [1024, 900, 0, 300, 1025], 3),
    (2, 32, 8, [4096, 2500], 16),
])
def test_paged_decode_attention_matches_oracle(B, hq, hkv, ctx, splits):
    if ctx is None:
        ctx_t, _, _, _, _ = cases.decode_batch(B, 100, 1024, 256, 0)
        ctx = ctx_t.tolist()
    q, pool, tables, ctxs = _decode_case(B, hq, hkv, ctx, seed=20, nan_tail=True)
    scale = 128 ** -0.5
    ref = ops.paged_decode_attention(q, pool[:, 0], pool[:, 1], tables, ctxs, scale)
    dpool = pool.to(DEV)
    out = K().paged_decode_attention(q.to(DEV), dpool[:, 0], dpool[:, 1], tables.to(DEV), ctxs.to(DEV), scale,
                                     num_splits=splits)
    assert not torch.isnan(out).any()
    close(out, ref)


def test_decode_attention_is_invariant_to_split_count():
    q, pool, tables, ctxs = _decode_case(3, 32, 8, [2000, 513, 64], seed=30)
    dpool = pool.to(DEV)
    outs = [K().paged_decode_attention(q.to(DEV), dpool[:, 0], dpool[:, 1], tables.to(DEV), ctxs.to(DEV), 0.088,
                                       num_splits=s) for s in (1, 2, 5, 32)]
    for o in outs[1:]:
        close(o, outs[0], atol=1e-2, rtol=1e-2)


# ------------------------------------------------------------------ prefill attention
@pytest.mark.parametrize("tensor_cores", [True, False])
def test_varlen_prefill_contiguous_matches_oracle(tensor_cores):
    lens = [1, 77, 300, 64, 129]
    hq, hkv = 16, 8
    T = sum(lens)
    qkv = torch.randn(T, (hq + 2 * hkv) * 128, generator=g(40)).to(torch.bfloat16)
    q = qkv[:, :hq * 128].view(T, hq, 128)
    k = qkv[:, hq * 128:(hq + hkv) * 128].view(T, hkv, 128)
    v = qkv[:, (hq + hkv) * 128:].view(T, hkv, 128)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    ref = ops.varlen_prefill_attention(q, k, v, cu, cu, 128 ** -0.5)
    d = qkv.to(DEV)
    out = K().prefill_attention(d[:, :hq * 128].view(T, hq, 128), d[:, hq * 128:(hq + hkv) * 128].view(T, hkv, 128),
                                d[:, (hq + hkv) * 128:].view(T, hkv, 128), cu.to(DEV), cu.to(DEV), max(lens),
                                128 ** -0.5, tensor_cores=tensor_cores)
    close(out, ref)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_paged_prefill_with_cached_prefix_matches_oracle(tensor_cores):
    """Chunked prefill / prefix-cache hit: new queries attend cached keys too
    (bottom-right causal alignment). Cache bytes past each sequence are NaN:
    neither kernel may let them reach the output."""
    hq, hkv, bs = 32, 8, 256
    cached = [256, 0, 512, 100, 0]
    new = [100, 50, 300, 1, 700]
    kv_len = [c + n for c, n in zip(cached, new)]
    need = [(x + bs - 1) // bs for x in kv_len]
    nblk = sum(need) + 1
    perm = torch.randperm(nblk, generator=g(41)).tolist()
    width = max(need)
    tables, j = [], 0
    for n in need:
        tables.append(perm[j:j + n] + [-1] * (width - n))
        j += n
    pool = torch.randn(nblk, 2, bs, hkv, 128, generator=g(42)).to(torch.bfloat16)
    for row, n in zip(tables, kv_len):  # stale bytes after the last key of each sequence
        last = row[(n - 1) // bs]
        pool[last, :, (n - 1) % bs + 1:] = float("nan")
    T = sum(new)
    q = torch.randn(T, hq, 128, generator=g(43)).to(torch.bfloat16)
    cu_q = torch.tensor([0] + torch.tensor(new).cumsum(0).tolist(), dtype=torch.int32)
    cu_k = torch.tensor([0] + torch.tensor(kv_len).cumsum(0).tolist(), dtype=torch.int32)
    bt = torch.tensor(tables, dtype=torch.int32)
    ref = ops.varlen_prefill_attention(q, pool[:, 0], pool[:, 1], cu_q, cu_k, 128 ** -0.5, bt)
    dpool = pool.to(DEV)
    out = K().prefill_attention(q.to(DEV), dpool[:, 0], dpool[:, 1], cu_q.to(DEV), cu_k.to(DEV), max(new),
                                128 ** -0.5, block_tables=bt.to(DEV), tensor_cores=tensor_cores)
    assert not out.isnan().any()
    close(out, ref)


# ------------------------------------------------------------------ sampler
def test_sampler_greedy_matches_argmax():
    logits = (torch.randn(512, 151936, generator=g(50)) * 3).to(torch.bfloat16)
    d = logits.to(DEV)
    seed = torch.zeros((), dtype=torch.int32, device=DEV)
    tok = K().sample(d, torch.zeros(512, dtype=torch.float32, device=DEV), seed)
    assert tok.dtype == torch.int64
    assert torch.equal(tok.cpu(), ops.greedy(logits))


def test_sampler_gumbel_matches_oracle_philox():
    B, V = 64, 3000
    logits = (torch.randn(B, V, generator=g(51)) * 2).to(torch.bfloat16)
    temps = torch.tensor([0.6, 1.0, 0.0, 1.3] * (B // 4), dtype=torch.float32)
    seed = 1234
    tok = K().sample(logits.to(DEV), temps.to(DEV), torch.tensor(seed, dtype=torch.int32, device=DEV)).cpu()
    scores = ops.gumbel_scores(logits, temps.clamp_min(1e-30), seed)
    ref = ops.sample(logits, temps, seed)
    for b in range(B):
        if tok[b] != ref[b]:  # only float near-ties may differ
            assert abs(scores[b, tok[b]].item() - scores[b, ref[b]].item()) < 1e-4, b


def test_sampler_gumbel_unaligned_noise_counters():
    """Rows whose global column counter does not start at a multiple of 4
    (vocab 3002 in rows of stride 3008, and a shard at column offset 1001):
    the 16-byte chunks take the per-column noise path, the aligned rows the
    4-columns-per-Philox-block path; both draw the oracle's noise."""
    B, V, S = 16, 3002, 3008
    full = (torch.randn(B, S, generator=g(54)) * 2).to(torch.bfloat16)
    logits = full[:, :V]
    temps = torch.tensor([0.6, 1.0, 1.3, 0.9] * (B // 4), dtype=torch.float32)
    seed = 4321
    dseed = torch.tensor(seed, dtype=torch.int32, device=DEV)
    tok = K().sample(full.to(DEV)[:, :V], temps.to(DEV), dseed).cpu()
    scores = ops.gumbel_scores(logits, temps, seed)
    ref = ops.sample(logits, temps, seed)
    for b in range(B):
        if tok[b] != ref[b]:
            assert abs(scores[b, tok[b]].item() - scores[b, ref[b]].item()) < 1e-4, b
    # the shard [1001, 3001) of the same rows, scored with its global columns
    off, n = 1001, 2000
    shard = full[:, off:off + n].contiguous().to(DEV)
    val = torch.empty(B, dtype=torch.float32, device=DEV)
    idx = torch.empty(B, dtype=torch.int64, device=DEV)
    K().sample_partial(shard, temps.to(DEV), dseed, off, V, val, idx)
    best = scores[:, off:off + n].argmax(-1) + off
    for b in range(B):
        got = int(idx[b])
        if got != int(best[b]):
            assert abs(scores[b, got].item() - scores[b, best[b]].item()) < 1e-4, b


def test_sampler_distribution_matches_softmax():
    V, N = 50, 20000
    logits = (torch.randn(V, generator=g(52)) * 4).to(torch.bfloat16)
    probs = torch.softmax(logits.float(), -1)
    tok = K().sample(logits.unsqueeze(0).expand(N, V).contiguous().to(DEV), torch.ones(N, device=DEV),
                     torch.tensor(7, dtype=torch.int32, device=DEV))
    freq = torch.bincount(tok.cpu(), minlength=V).float() / N
    assert (freq - probs).abs().max().item() < 0.01


def test_sharded_sampling_equals_full_row():
    B, V, world = 8, 4096, 4
    logits = torch.randn(B, V, generator=g(53)).to(torch.bfloat16).to(DEV)
    temps = torch.tensor([0.0, 0.7] * 4, dtype=torch.float32, device=DEV)
    seed = torch.tensor(99, dtype=torch.int32, device=DEV)
    full = K().sample(logits, temps, seed)
    vals = torch.empty(world, B, dtype=torch.float32, device=DEV)
    idxs = torch.empty(world, B, dtype=torch.int64, device=DEV)
    shard = V // world
    for r in range(world):
        K().sample_partial(logits[:, r * shard:(r + 1) * shard].contiguous(), temps, seed, r * shard, V, vals[r], idxs[r])
    out = torch.empty(B, dtype=torch.int64, device=DEV)
    assert torch.equal(K().sample_combine(vals, idxs, out), full)


# ------------------------------------------------------------------ device-side bounds checks
def test_out_of_range_block_id_is_reported_not_read():
    from kavor_b200 import _lib as L

    q, pool, tables, ctxs = _decode_case(2, 32, 8, [300, 300], seed=60)
    tables[1, 1] = pool.shape[0] + 5  # points past the pool
    dpool = pool.to(DEV)
    K().paged_decode_attention(q.to(DEV), dpool[:, 0], dpool[:, 1], tables.to(DEV), ctxs.to(DEV), 0.088, num_splits=1)
    assert L.device_error(clear=True) & 1
