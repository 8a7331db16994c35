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


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")
@pytest.mark.parametrize("splits", [4, 0])
def test_no_alloc_decode_matches_workspace_entry_point_twice(splits):
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
    assert _lib.device_error(clear=True) == 0


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")
def test_no_alloc_decode_rejects_scratch_beyond_its_limit():
    from kavor_b200 import _lib

    lib = _lib.load()
    q, pool, tables, ctx = _case(2)
    out = torch.empty_like(q)
    # 3 sequences x 32 heads x 2000 splits x 516 B = 99 MB > 8 MiB
    rc = _call_no_alloc(lib, q, pool, tables, ctx, out, 2000)
    assert rc == -3
    assert b"built-in area" in lib.kvb_last_error()
