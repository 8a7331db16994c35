"""kvb_paged_decode_attn_no_alloc: the decode attention for callers that cannot
hand the library scratch memory (inputs and outputs only). Called through the
C ABI and compared with the regular entry point, which gets a caller-provided
workspace, on two calls in a row (the built-in scratch keeps the previous
call's contents, so the second call must not depend on them). Kept in its own
file, collected last."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(seed=0):
    g = torch.Generator().manual_seed(seed)
    B, hq, hkv, hd, bs = 3, 32, 8, 128, 256
    ctx = [2000, 513, 64]
    need = [(c + bs - 1) // bs for c in ctx]
    nblk = sum(need) + 2
    perm = torch.randperm(nblk, generator=g).tolist()
    tables, k = [], 0
    for n in need:
        tables.append(perm[k:k + n] + [-1] * (max(need) - n))
        k += n
    pool = torch.randn(nblk, 2, bs, hkv, hd, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(B, hq, hd, generator=g).to(torch.bfloat16).to(DEV)
    return q, pool, torch.tensor(tables, dtype=torch.int32, device=DEV), torch.tensor(ctx, dtype=torch.int32, device=DEV)


def _call_no_alloc(lib, q, pool, tables, ctx, out, splits):
    k, v = pool[:, 0], pool[:, 1]
    return lib.kvb_paged_decode_attn_no_alloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.size(0), k.stride(0), k.size(1),
        tables.data_ptr(), tables.stride(0), tables.shape[1], ctx.data_ptr(), out.data_ptr(), out.stride(0),
        out.stride(1), q.shape[0], q.shape[1], k.size(2), q.shape[2], ctypes.c_float(128 ** -0.5), splits,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _oracle(q, pool, tables, ctx):
    from oracle import ops

    return ops.paged_decode_attention(q.cpu(), pool[:, 0].cpu(), pool[:, 1].cpu(), tables.cpu(), ctx.cpu(),
                                      128 ** -0.5)


# 3 sequences x 32 query heads = 96 partial rows of 516 B (128 fp32 values and
# a log-sum-exp) per split: 169 splits use 8,371,584 B of the 8 MiB area, 170
# would need 8,421,120 B
SPLITS_AT_LIMIT = 169


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")
@pytest.mark.parametrize("splits", [1, 4, 0, SPLITS_AT_LIMIT])
def test_no_alloc_decode_matches_workspace_entry_point_twice(splits):
    """splits 1 uses no scratch, 0 lets the library choose, 169 fills the
    built-in area up to its last whole split; each output equals the
    workspace entry point's within the attention tolerance, and the oracle's."""
    from kavor_b200 import _kernels as K
    from kavor_b200 import _lib

    lib = _lib.load()
    for seed in (0, 1):  # two calls in a row, different inputs
        q, pool, tables, ctx = _case(seed)
        ref = K.paged_decode_attention(q, pool[:, 0], pool[:, 1], tables, ctx, 128 ** -0.5, num_splits=splits)
        out = torch.full_like(q, float("nan"))
        rc = _call_no_alloc(lib, q, pool, tables, ctx, out, splits)
        assert rc == 0, lib.kvb_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=1e-2)
        torch.testing.assert_close(out.float().cpu(), _oracle(q, pool, tables, ctx).float(), atol=2e-2, rtol=1e-2)
    assert _lib.device_error(clear=True) == 0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")
@pytest.mark.parametrize("splits", [SPLITS_AT_LIMIT + 1, 2000])
def test_no_alloc_decode_rejects_scratch_beyond_its_limit(splits):
    from kavor_b200 import _lib

    lib = _lib.load()
    q, pool, tables, ctx = _case(2)
    out = torch.empty_like(q)
    rc = _call_no_alloc(lib, q, pool, tables, ctx, out, splits)
    assert rc == -3
    assert b"built-in area" in lib.kvb_last_error()
