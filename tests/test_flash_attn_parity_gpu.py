"""Attention parity against the third-party library the reference calls
(flash-attn 2.8.3, flash_attention_kvcache.py:76-83), run on the same GPU on
identical seeded inputs: the paged decode call
flash_attn_with_kvcache(q[:, None], k_cache, v_cache, cache_seqlens, block_table,
causal=True) and the varlen prefill call flash_attn_varlen_func(...,
causal=True[, block_table]) against kvb_paged_decode_attn / kvb_prefill_attn.
The library is only run, as the reference runs it; the test skips when it is
not installed or has no kernel for this GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def fa():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    fa = pytest.importorskip("flash_attn")
    q = torch.randn(1, 1, 8, 128, device=DEV, dtype=torch.bfloat16)
    kc = torch.randn(1, 256, 8, 128, device=DEV, dtype=torch.bfloat16)
    try:
        fa.flash_attn_with_kvcache(q, kc, kc, cache_seqlens=torch.ones(1, dtype=torch.int32, device=DEV),
                                   block_table=torch.zeros(1, 1, dtype=torch.int32, device=DEV), causal=True)
        torch.cuda.synchronize()
    except RuntimeError as e:  # e.g. no kernel image for this architecture
        pytest.skip(f"flash-attn does not run on this GPU: {e}")
    return fa


def _pages(ctx, hkv, bs, seed):
    g = torch.Generator().manual_seed(seed)
    need = [(c + bs - 1) // bs for c in ctx]
    nblk = sum(need) + 2
    perm = torch.randperm(nblk, generator=g).tolist()
    width = max(need)
    tables, j = [], 0
    for n in need:
        tables.append(perm[j:j + n] + [0] * (width - n))  # flash-attn wants valid ids in the padding too
        j += n
    pool = torch.randn(nblk, 2, bs, hkv, 128, generator=g).to(torch.bfloat16).to(DEV)
    return pool, torch.tensor(tables, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (4, 1), (16, 8)])
def test_decode_matches_flash_attn(fa, hq, hkv):
    from kavor_b200 import _kernels as K

    ctx = [1, 255, 256, 257, 1024, 700, 3000, 64]
    B = len(ctx)
    pool, bt = _pages(ctx, hkv, 256, seed=hq)
    q = torch.randn(B, hq, 128, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).to(DEV)
    cl = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    ref = fa.flash_attn_with_kvcache(q.unsqueeze(1), pool[:, 0], pool[:, 1], cache_seqlens=cl, block_table=bt,
                                     softmax_scale=128 ** -0.5, causal=True).squeeze(1)
    ours = K.paged_decode_attention(q, pool[:, 0], pool[:, 1], bt, cl, 128 ** -0.5)
    torch.testing.assert_close(ours.float(), ref.float(), atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_varlen_prefill_matches_flash_attn(fa, tensor_cores):
    from kavor_b200 import _kernels as K

    lens = [1, 77, 300, 129, 1000]
    hq, hkv, T = 32, 8, sum(lens)
    g = torch.Generator().manual_seed(11)
    q = torch.randn(T, hq, 128, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(T, hkv, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(T, hkv, 128, generator=g).to(torch.bfloat16).to(DEV)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    ref = fa.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=128 ** -0.5, causal=True)
    ours = K.prefill_attention(q, k, v, cu, cu, max(lens), 128 ** -0.5, tensor_cores=tensor_cores)
    torch.testing.assert_close(ours.float(), ref.float(), atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_paged_prefill_with_prefix_matches_flash_attn(fa, tensor_cores):
    from kavor_b200 import _kernels as K

    cached, new = [256, 0, 512, 100], [100, 50, 300, 1]
    kv_len = [c + n for c, n in zip(cached, new)]
    hq, hkv = 32, 8
    pool, bt = _pages(kv_len, hkv, 256, seed=3)
    T = sum(new)
    q = torch.randn(T, hq, 128, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    cu_q = torch.tensor([0] + torch.tensor(new).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0] + torch.tensor(kv_len).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    ref = fa.flash_attn_varlen_func(q, pool[:, 0], pool[:, 1], cu_q, cu_k, max(new), max(kv_len),
                                    softmax_scale=128 ** -0.5, causal=True, block_table=bt)
    ours = K.prefill_attention(q, pool[:, 0], pool[:, 1], cu_q, cu_k, max(new), 128 ** -0.5, block_tables=bt,
                               tensor_cores=tensor_cores)
    torch.testing.assert_close(ours.float(), ref.float(), atol=2e-2, rtol=1e-2)
