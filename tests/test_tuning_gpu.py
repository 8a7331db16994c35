"""GEMM tuning options that are off by default, against the same references as
test_gemm_gpu.py: K splits whose cluster size is not a power of two (the
reduction deals the tile's sixteen 8-feature groups unevenly over the ranks)
and the L2 prefetch of the weight stream (kvb_gemm_set_l2_prefetch)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from kavor_b200 import _kernels as K_
    from kavor_b200 import _lib

    _lib.load()
    _lib.device_error(clear=True)
    yield
    K_.gemm_set_l2_prefetch(0)
    assert _lib.device_error(clear=True) == 0


def _inputs(M, N, K, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("M,N,K,splits", [
    (256, 6144, 4096, 3), (64, 4096, 4096, 5), (16, 4096, 12288, 6), (256, 4096, 4096, 7), (1, 768, 4096, 10),
    (100, 1000, 1536, 3),
])
def test_gemm_non_power_of_two_cluster_split(M, N, K, splits):
    from kavor_b200 import _kernels as K_

    assert K_.gemm_plan(M, N, K, splits)["splits"] == splits
    x, w = _inputs(M, N, K)
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm(x, w, out=y, splits=splits)
    torch.testing.assert_close(y.float(), x.float() @ w.float().t(), atol=1e-2, rtol=1e-2)
    assert torch.equal(y, K_.gemm(x, w, splits=splits))  # fixed summation order


@pytest.mark.parametrize("splits", [3, 6])
def test_gated_gemm_non_power_of_two_cluster_split(splits):
    from kavor_b200 import _kernels as K_

    M, inter, K = 64, 1536, 4096
    x, w = _inputs(M, 2 * inter, K, seed=3)
    out = torch.full((M, inter), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm_silu(x, w, out=out, splits=splits)
    ref32 = x.float() @ w.float().t()
    g, u = ref32[:, :inter].to(torch.bfloat16).float(), ref32[:, inter:].to(torch.bfloat16).float()
    torch.testing.assert_close(out.float(), torch.nn.functional.silu(g) * u, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("ksteps", [2, 8, 64])
def test_gemm_l2_prefetch_leaves_results_unchanged(ksteps):
    """The prefetch only moves weight bytes into L2 early: bit-identical
    outputs, persistent and cluster schedules, plain and gated."""
    from kavor_b200 import _kernels as K_

    cases = [(256, 6144, 4096, 0, False), (7, 768, 4096, 1, False), (64, 4096, 12288, 4, False),
             (256, 3072, 4096, 0, True)]
    for M, N, K, splits, gated in cases:
        x, w = _inputs(M, (2 if gated else 1) * N, K, seed=5)
        fn = K_.gemm_silu if gated else K_.gemm
        K_.gemm_set_l2_prefetch(0)
        ref = fn(x, w, splits=splits)
        K_.gemm_set_l2_prefetch(ksteps)
        assert torch.equal(fn(x, w, splits=splits), ref), (M, N, K, splits, gated)
