"""tcgen05 GEMM (kvb_gemm_bf16) parity: y = x w^T against an fp32 reference and
against cuBLAS (F.linear, the reference's GEMM), over decode and prefill shapes
of Qwen3 projections at TP 1..8, ragged M and N, forced split-K, determinism."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from kavor_b200 import _lib

    _lib.load()
    _lib.device_error(clear=True)
    yield
    assert _lib.device_error(clear=True) == 0


def _inputs(M, N, K, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("M,N,K,splits", [
    (1, 768, 4096, 0), (7, 6144, 4096, 0), (16, 4096, 512, 0), (33, 3072, 4096, 0), (64, 4096, 1536, 0),
    (100, 1000, 4096, 0), (128, 4096, 4096, 1), (200, 4096, 12288, 0), (256, 6144, 4096, 0),
    (256, 4096, 4096, 4), (64, 4096, 4096, 16), (16, 4096, 1536, 2), (256, 18992, 4096, 0), (300, 2048, 1024, 0), (1024, 1024, 4096, 0),
    (256, 24576, 4096, 1), (256, 24576, 4096, 2), (2048, 4096, 4096, 0),
])
def test_gemm_matches_fp32_reference_and_cublas(M, N, K, splits):
    from kavor_b200 import _kernels as K_

    x, w = _inputs(M, N, K)
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm(x, w, out=y, splits=splits)
    ref = x.float() @ w.float().t()
    torch.testing.assert_close(y.float(), ref, atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(y.float(), F.linear(x, w).float(), atol=1e-2, rtol=1e-2)


def test_gemm_split_k_is_deterministic():
    from kavor_b200 import _kernels as K_

    x, w = _inputs(64, 4096, 12288, seed=1)
    a = K_.gemm(x, w, splits=8)
    b = K_.gemm(x, w, splits=8)
    assert torch.equal(a, b)
    c = K_.gemm(x, w, splits=1)
    torch.testing.assert_close(a.float(), c.float(), atol=1e-2, rtol=1e-2)



def test_gemm_back_to_back_splits_of_different_tile_counts():
    """Split-K (cluster) and persistent calls of different tile counts, plain
    and gated, back to back into NaN-filled outputs: no call depends on state
    a previous call left behind."""
    from kavor_b200 import _kernels as K_

    shapes = [(256, 6144, 4096, 0, False), (256, 24576, 4096, 2, False), (64, 1536, 4096, 4, True),
              (256, 12288, 4096, 2, True), (16, 151936 // 8, 4096, 16, False), (256, 24576, 4096, 1, False), (1, 768, 4096, 8, False)]
    for i, (M, N, K, splits, gated) in enumerate(shapes * 2):
        x, w = _inputs(M, (2 if gated else 1) * N, K, seed=10 + i)
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
        ref32 = x.float() @ w.float().t()
        if gated:
            K_.gemm_silu(x, w, out=out, splits=splits)
            g, u = ref32[:, :N].to(torch.bfloat16).float(), ref32[:, N:].to(torch.bfloat16).float()
            ref = torch.nn.functional.silu(g) * u
            torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
        else:
            K_.gemm(x, w, out=out, splits=splits)
            torch.testing.assert_close(out.float(), ref32, atol=1e-2, rtol=1e-2)


def test_gemm_writes_into_strided_output_rows():
    from kavor_b200 import _kernels as K_

    x, w = _inputs(40, 512, 1024, seed=2)
    big = torch.zeros(40, 1024, dtype=torch.bfloat16, device=DEV)
    K_.gemm(x, w, out=big[:, 256:768])
    torch.testing.assert_close(big[:, 256:768].float(), (x.float() @ w.float().t()), atol=1e-2, rtol=1e-2)
    assert big[:, :256].abs().sum() == 0 and big[:, 768:].abs().sum() == 0


@pytest.mark.parametrize("M,inter,K,splits", [
    (1, 1536, 4096, 0), (16, 3072, 4096, 0), (64, 1536, 4096, 4), (256, 12288, 4096, 0), (300, 1000, 1024, 0),
    (256, 3072, 4096, 0), (256, 1536, 4096, 8), (1, 1536, 4096, 16),
])
def test_gemm_silu_matches_projection_then_silu_mul(M, inter, K, splits):
    """Fused gate-up + SiLU*mul == bf16(x Wg^T), bf16(x Wu^T), then SiluAndMul
    (the reference's two steps and rounding points)."""
    from kavor_b200 import _kernels as K_
    from oracle import ops

    x, w = _inputs(M, 2 * inter, K, seed=3)
    y = torch.full((M, inter), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm_silu(x, w, out=y, splits=splits)
    gu = (x.float() @ w.float().t()).to(torch.bfloat16)
    ref = ops.silu_mul(gu.cpu()).to(DEV)
    torch.testing.assert_close(y.float(), ref.float(), atol=2e-2, rtol=2e-2)
