"""CTA-pair GEMM (kvb_gemm_pair_bf16, tcgen05 cta_group::2) against an fp32
reference and cuBLAS over decode and prefill shapes of the Qwen3 projections,
ragged M and N, forced K splits, NaN-filled outputs and determinism."""
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
    (1, 768, 4096, 0), (7, 6144, 4096, 0), (64, 4096, 512, 0), (100, 1000, 4096, 0), (128, 4096, 4096, 1),
    (256, 6144, 4096, 0), (256, 4096, 12288, 0), (256, 4096, 4096, 3), (33, 3072, 4096, 5), (256, 768, 4096, 8),
    (300, 2048, 1024, 0), (256, 18992, 4096, 0),
])
def test_gemm_pair_matches_fp32_reference_and_cublas(M, N, K, splits):
    from kavor_b200 import _kernels as K_

    x, w = _inputs(M, N, K)
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm_pair(x, w, out=y, splits=splits)
    torch.testing.assert_close(y.float(), x.float() @ w.float().t(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(y.float(), F.linear(x, w).float(), atol=1e-2, rtol=1e-2)


def test_gemm_pair_split_is_deterministic():
    from kavor_b200 import _kernels as K_

    x, w = _inputs(256, 4096, 12288, seed=1)
    a = K_.gemm_pair(x, w, splits=4)
    assert torch.equal(a, K_.gemm_pair(x, w, splits=4))
    torch.testing.assert_close(a.float(), K_.gemm_pair(x, w, splits=1).float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("M,inter,K,splits", [(1, 1536, 4096, 0), (64, 3072, 1024, 1), (100, 1000, 4096, 0),
                                              (256, 12288, 4096, 1), (256, 12288, 4096, 3), (300, 1536, 4096, 0),
                                              (256, 1536, 4096, 6), (33, 768, 4096, 5)])
def test_gemm_pair_silu_matches_the_rounded_reference(M, inter, K, splits):
    """bf16(silu(bf16(x w_gate^T)) * bf16(x w_up^T)), the reference's rounding points."""
    from kavor_b200 import _kernels as K_

    x, w = _inputs(M, 2 * inter, K, seed=7)
    out = torch.full((M, inter), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm_pair_silu(x, w, out=out, splits=splits)
    ref32 = x.float() @ w.float().t()
    g, u = ref32[:, :inter].to(torch.bfloat16).float(), ref32[:, inter:].to(torch.bfloat16).float()
    torch.testing.assert_close(out.float(), F.silu(g) * u, atol=2e-2, rtol=2e-2)
