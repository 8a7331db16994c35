"""Host-side plan of the stream-K GEMM (no GPU: the planner assumes the B200's
148 SMs when it cannot query a device): every pair gets a non-empty range, the
workspace query bounds what any plan of the shape needs, and the plan
override is validated."""
import ctypes

import pytest

SHAPES = [(1, 6144, 4096), (16, 4096, 4096), (64, 24576, 4096), (100, 1000, 4096), (256, 6144, 4096),
          (256, 4096, 12288), (256, 151936, 4096), (256, 4096, 512), (300, 2048, 1024), (5, 200, 64)]


@pytest.fixture(scope="module")
def K():
    from kavor_b200 import _kernels, _lib, build

    build.build()
    _lib.load()
    return _kernels


@pytest.mark.parametrize("M,N,Kd", SHAPES)
def test_plan_covers_the_shape(K, M, N, Kd):
    for gated in (False, True):
        p = K.gemm_sk_plan(M, N, Kd, gated)
        assert p["mt"] in (16, 32, 64, 128, 256) and (p["mt"] >= min(M, 256) or p["mt"] == 128)
        assert 1 <= p["pairs"] <= 74 and p["pairs"] <= p["tiles"] * p["kb"]  # every range non-empty
        assert p["kb"] * 64 * (2 if p["mt"] >= 128 else 3) >= Kd  # the K steps reach K
        rows = 128 if gated else 256
        assert p["tiles"] * rows >= N


@pytest.mark.parametrize("M,N,Kd", SHAPES)
def test_workspace_query_bounds_every_forced_plan(K, M, N, Kd):
    need_max = 0
    try:
        for mt in (16, 32, 64, 128, 256):
            for pairs in (1, 16, 48, 74):
                K.gemm_sk_set_plan(mt, pairs)
                p = K.gemm_sk_plan(M, N, Kd)
                need_max = max(need_max, 1024 + p["pairs"] * 2 * 128 * p["mt"] * 4)
    finally:
        K.gemm_sk_set_plan(0, 0)
    assert K.gemm_sk_workspace_bytes(M, N, Kd) >= need_max


def test_plan_override_is_validated(K):
    from kavor_b200 import _lib

    lib = _lib.load()
    assert lib.kvb_gemm_sk_set_plan(48, 0) < 0  # not a token tile
    assert lib.kvb_gemm_sk_set_plan(0, 1000) < 0
    assert b"kvb_gemm_sk_set_plan" in lib.kvb_last_error()
    assert lib.kvb_gemm_sk_set_plan(0, 0) == 0


def test_entry_points_reject_bad_arguments_on_the_host(K):
    from kavor_b200 import _lib

    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.kvb_gemm_sk_workspace_size(0, 4096, 4096, 0, ctypes.byref(n)) == 0 and n.value == 0
    # K not a multiple of 64 (checked before any launch)
    rc = lib.kvb_gemm_sk_bf16(16, 4104, 16, 4104, 16, 4096, 8, 4096, 4104, 16, 1 << 20, None)
    assert rc == -2 and b"multiple of 64" in lib.kvb_last_error()
    # no workspace
    rc = lib.kvb_gemm_sk_bf16(16, 4096, 16, 4096, 16, 4096, 8, 4096, 4096, None, 0, None)
    assert rc == -3 and b"workspace" in lib.kvb_last_error()
