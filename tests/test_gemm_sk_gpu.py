"""Stream-K CTA-pair GEMM (kvb_gemm_sk_bf16 / kvb_gemm_sk_silu_bf16) against
an fp32 reference and cuBLAS: decode and ragged shapes of the Qwen3
projections (M from 1 to 300 tokens, N and K not multiples of the tiles),
tiles cut between pairs (partials summed by the owner in K order), the fused
gate-up + SiLU form, determinism, several shapes sharing one workspace, and
CUDA-graph replay."""
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


SHAPES = [
    (1, 768, 4096), (7, 6144, 4096), (16, 4096, 4096), (33, 3072, 4096), (64, 4096, 512), (100, 1000, 4096),
    (128, 4096, 4096), (200, 6144, 4096), (256, 6144, 4096), (256, 4096, 12288), (256, 4096, 512),
    (256, 18992, 4096), (256, 768, 4096), (300, 2048, 1024), (5, 200, 64), (256, 4096, 1536), (1, 151936, 4096),
    (256, 151936, 4096),  # the default path's LM head at the headline batch: several whole tiles per pair
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_sk_matches_fp32_reference_and_cublas(M, N, K):
    from kavor_b200 import _kernels as K_

    x, w = _inputs(M, N, K)
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm_sk(x, w, out=y)
    torch.testing.assert_close(y.float(), x.float() @ w.float().t(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(y.float(), F.linear(x, w).float(), atol=1e-2, rtol=1e-2)


GATED = [(1, 1536, 4096), (64, 3072, 1024), (100, 1000, 4096), (256, 12288, 4096), (256, 1536, 4096),
         (33, 768, 4096), (300, 1536, 4096), (16, 12288, 4096)]


@pytest.mark.parametrize("M,inter,K", GATED)
def test_gemm_sk_silu_matches_the_rounded_reference(M, inter, K):
    """bf16(silu(bf16(x w_gate^T)) * bf16(x w_up^T)), the reference's rounding points."""
    from kavor_b200 import _kernels as K_

    x, w = _inputs(M, 2 * inter, K, seed=7)
    out = torch.full((M, inter), float("nan"), dtype=torch.bfloat16, device=DEV)
    K_.gemm_sk_silu(x, w, out=out)
    ref32 = x.float() @ w.float().t()
    g, u = ref32[:, :inter].to(torch.bfloat16).float(), ref32[:, inter:].to(torch.bfloat16).float()
    torch.testing.assert_close(out.float(), F.silu(g) * u, atol=2e-2, rtol=2e-2)


def test_gemm_sk_is_deterministic_and_leaves_the_workspace_clean():
    """Same inputs, same bits; the hand-off flags are zero after every launch,
    so the next shape that shares the workspace sees none of them."""
    from kavor_b200 import _kernels as K_

    shapes = [(256, 6144, 4096), (256, 4096, 4096), (256, 4096, 12288), (64, 3072, 4096)]
    runs = []
    for rep in range(2):
        outs = []
        for i, (M, N, K) in enumerate(shapes):
            x, w = _inputs(M, N, K, seed=i)
            outs.append(K_.gemm_sk(x, w))
        runs.append(outs)
        torch.cuda.synchronize()
        ws = K_.GEMM_WORKSPACE.buf[torch.cuda.current_device()]
        assert int(ws[:1024].sum()) == 0  # the flags (2 per pair, at most 128 pairs) lead the workspace
    for a, b in zip(*runs):
        assert torch.equal(a, b)
    for (M, N, K), y, i in zip(shapes, runs[0], range(len(shapes))):
        x, w = _inputs(M, N, K, seed=i)
        torch.testing.assert_close(y.float(), x.float() @ w.float().t(), atol=1e-2, rtol=1e-2)


def test_gemm_sk_first_call_in_a_fresh_process():
    """A decode-batch shape whose plan uses a smaller token tile than the batch
    (256 tokens as two 128-token tiles) as the process's first launch: every
    kernel variant a plan picks is set up before it is launched."""
    import subprocess
    import sys
    from pathlib import Path

    code = ("import torch; from kavor_b200 import _kernels as K; "
            "x = torch.randn(256, 4096, device='cuda').to(torch.bfloat16); "
            "w = (torch.randn(6144, 4096, device='cuda') * 0.02).to(torch.bfloat16); "
            "y = K.gemm_sk(x, w); torch.cuda.synchronize(); "
            "assert (y.float() - x.float() @ w.float().t()).abs().max().item() < 5e-2")
    root = str(Path(__file__).resolve().parents[1])
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]


def test_gemm_sk_graph_replay():
    """Three projections captured in one CUDA graph, replayed with new inputs."""
    from kavor_b200 import _kernels as K_

    M = 256
    x = torch.empty(M, 4096, dtype=torch.bfloat16, device=DEV)
    _, wq = _inputs(M, 6144, 4096, seed=1)
    _, wgu = _inputs(M, 2 * 12288, 4096, seed=2)
    _, wd = _inputs(M, 4096, 12288, seed=3)
    K_.gemm_sk(x.normal_(), wq)  # workspace reserved before capture
    K_.gemm_sk_silu(x, wgu)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        q = K_.gemm_sk(x, wq)
        h = K_.gemm_sk_silu(x, wgu)
        d = K_.gemm_sk(h, wd)
    for seed in (4, 5):
        x.copy_(torch.randn(M, 4096, generator=torch.Generator(device=DEV).manual_seed(seed), device=DEV))
        g.replay()
        torch.cuda.synchronize()
        torch.testing.assert_close(q.float(), x.float() @ wq.float().t(), atol=1e-2, rtol=1e-2)
        ref = x.float() @ wgu.float().t()
        hh = (F.silu(ref[:, :12288].to(torch.bfloat16).float()) * ref[:, 12288:].to(torch.bfloat16).float())
        torch.testing.assert_close(h.float(), hh, atol=2e-2, rtol=2e-2)
        torch.testing.assert_close(d.float(), h.float() @ wd.float().t(), atol=2e-2, rtol=2e-2)
