"""The C-ABI library builds, loads and exports exactly the entry points that
include/kavor_b200.h declares (no GPU needed: only host-side argument checks
are exercised, nothing is launched)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    from kavor_b200 import _lib, build

    build.build()
    return _lib.load()


def _declared():
    text = (ROOT / "include" / "kavor_b200.h").read_text()
    return set(re.findall(r"^(?:int|const char\*)\s+(kvb_\w+)\(", text, flags=re.M))


def test_header_and_binding_agree():
    from kavor_b200 import _lib

    assert _declared() == set(_lib.exported_symbols())


def test_every_declared_symbol_is_exported(lib):
    for name in _declared():
        assert hasattr(lib, name), name


def test_only_the_api_is_exported(lib):
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "kavor_b200" / "libkavor_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == _declared()


def test_version_and_host_side_validation(lib):
    assert lib.kvb_version() == 100
    # invalid sizes are rejected on the host with a negative status and a message
    rc = lib.kvb_store_kv(None, 0, None, 0, None, None, 0, 0, 256, 8, 128, None, -1, None)
    assert rc < 0
    assert b"kvb_store_kv" in lib.kvb_last_error()
    rc = lib.kvb_paged_decode_attn(None, 0, 0, None, None, 10, 0, 256, None, 0, 4, None, None, 0, 0,
                                   4, 32, 8, 64, 0.1, 0, None, 0, None)
    assert rc < 0 and b"head_dim" in lib.kvb_last_error()
    n = ctypes.c_size_t(123)
    assert lib.kvb_paged_decode_attn_workspace_size(256, 32, 8, 128, 5, 256, 1, ctypes.byref(n)) == 0
    assert n.value == 0  # a single split needs no scratch
    assert lib.kvb_paged_decode_attn_workspace_size(1, 32, 8, 128, 5, 256, 4, ctypes.byref(n)) == 0
    assert n.value == 1 * 32 * 4 * (128 + 1) * 4


def test_ops_raise_without_a_cuda_tensor():
    import torch

    from kavor_b200 import _kernels as K

    x = torch.zeros(4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        K.rmsnorm(x, torch.ones(128, dtype=torch.bfloat16), 1e-6)


def test_gemm_plans_are_consistent(lib):
    """Host-side GEMM planning (no launch): every plan covers the problem, fits
    the SM budget (persistent) or forms whole clusters (split K), and needs no
    scratch memory."""
    import math

    from kavor_b200 import _kernels as K

    for M in (1, 7, 16, 64, 100, 256, 300, 2048, 16384):
        for N, Kd in ((768, 4096), (6144, 4096), (4096, 512), (4096, 12288), (151936, 4096), (1000, 1024)):
            p = K.gemm_plan(M, N, Kd)
            assert p["mt"] in (16, 32, 64, 128, 256)
            n_tiles, m_tiles = math.ceil(N / 128), math.ceil(M / p["mt"])
            kb = math.ceil(Kd / 64)
            assert 1 <= p["splits"] <= kb
            assert p["units"] == n_tiles * m_tiles * p["splits"]
            if p["splits"] == 1:  # persistent CTAs
                assert 1 <= p["grid"] <= min(p["units"], 2 * 148)
            else:  # one CTA per unit, clusters of `splits` CTAs along K, no empty part
                assert p["splits"] in (2, 4, 8, 16) and p["grid"] == p["units"]
                assert (p["splits"] - 1) * math.ceil(kb / p["splits"]) < kb
            assert K.gemm_workspace_bytes(M, N, Kd) == 0  # the split reduces through distributed shared memory


def test_gemm_forced_splits_of_any_cluster_size(lib):
    """A requested K split of 1..16 CTAs is taken exactly when every part gets
    K-steps (ceil(kb / C) per part, the last one non-empty); the reduction fits
    the stage ring of some token tile at every such split for these shapes
    (the 128-token tile and smaller take any C), otherwise the cost model's
    own plan is used."""
    import math

    from kavor_b200 import _kernels as K

    for splits in range(1, 17):
        for M, N, Kd in ((256, 6144, 4096), (64, 4096, 12288), (1, 768, 4096), (100, 1000, 1536)):
            p = K.gemm_plan(M, N, Kd, splits)
            kb = math.ceil(Kd / 64)
            if (splits - 1) * math.ceil(kb / splits) < kb:
                assert p["splits"] == splits, (M, N, Kd, splits, p)
                assert p["units"] == math.ceil(N / 128) * math.ceil(M / p["mt"]) * splits
                assert splits == 1 or (p["grid"] == p["units"] and p["units"] % splits == 0)
            else:
                assert p == K.gemm_plan(M, N, Kd)


def test_gemm_pair_plans(lib):
    """Host-side plan of the CTA-pair GEMM (no launch): token tile 64 / 128 /
    256 by batch, 256-row weight tiles, K splits that keep each tile's
    2 x splits CTAs within one CTA per SM, every part non-empty."""
    import math

    from kavor_b200 import _kernels as K

    for M in (1, 7, 64, 65, 128, 200, 256, 300, 2048):
        for N, Kd in ((768, 4096), (6144, 4096), (4096, 512), (4096, 12288), (151936, 4096), (1000, 1024)):
            p = K.gemm_pair_plan(M, N, Kd)
            mt = 64 if M <= 64 else (128 if M <= 128 else 256)
            tiles = math.ceil(N / 256) * math.ceil(M / mt)
            kb = math.ceil(Kd / 64)
            assert p["mt"] == mt and p["tiles"] == tiles and p["ctas"] == 2 * tiles * p["splits"]
            assert 1 <= p["splits"] <= 8 and (p["splits"] - 1) * math.ceil(kb / p["splits"]) < kb
            # no other valid split has fewer K-steps on the critical path (waves of 148 CTAs, each paying
            # 4 steps' worth of reduction when split)
            def cost(v):
                return math.ceil(2 * tiles * v / 148) * (math.ceil(kb / v) + (4 if v > 1 else 0))
            for v in range(2, 9):
                if (v - 1) * math.ceil(kb / v) < kb and v <= kb:
                    assert cost(p["splits"]) <= cost(v), (M, N, Kd, p, v)
    assert K.gemm_pair_plan(256, 6144, 4096)["splits"] == 3     # Qwen3-8B QKV, 256 tokens: 144 CTAs, one wave
    assert K.gemm_pair_plan(256, 24576, 4096)["splits"] == 3    # gate-up: 4 waves x (22 + 4) steps beat 2 x 64
    assert K.gemm_pair_plan(256, 151936, 4096)["splits"] == 1   # LM head: 9 waves unsplit
    assert K.gemm_pair_plan(256, 6144, 4096, splits=5)["splits"] == 5
    for M, inter in ((1, 1536), (100, 3072), (256, 12288), (300, 1000)):  # gated: 128-feature tiles
        mt = 64 if M <= 64 else (128 if M <= 128 else 256)
        p = K.gemm_pair_plan(M, inter, 4096, gated=True)
        assert p["tiles"] == math.ceil(inter / 128) * math.ceil(M / mt) and p["mt"] == mt
        assert p["ctas"] == 2 * p["tiles"] * p["splits"]
    assert K.gemm_pair_plan(256, 1536, 4096, gated=True)["splits"] == 6   # TP=8 gate-up: 12 tiles x 6 x 2 = 144 CTAs


def test_allreduce_plan_matches_the_documented_choice(lib):
    """Host-side mode choice of the fused all-reduce (no launch): peer one-shot
    at 2 ranks, switch one-shot below 8 rows per rank and switch two-shot from
    there with a multicast mapping at 4 and 8 ranks, peer two-shot without one
    when the one-shot would read more than 8 MiB per rank; explicit modes win."""
    from kavor_b200.layers.allreduce import allreduce_plan

    H = 4096
    for world in (2, 4, 8):
        for tokens in (1, 7, 8 * world - 1, 8 * world, 256, 4096):
            for mc in (False, True):
                p = allreduce_plan(world, mc, tokens, H)
                if mc and world > 2:
                    assert p["switch"] == (2 if tokens >= 8 * world else 1), (world, tokens)
                else:
                    assert p["switch"] == 0
                    assert p["peer_two_shot"] == int(world > 2 and tokens * H * 2 * world > 8 << 20)
    assert allreduce_plan(2, False, 5, H, mode=2) == {"peer_two_shot": 1, "switch": 0}
    assert allreduce_plan(8, True, 5, H, mode=4)["switch"] == 2
    assert allreduce_plan(8, True, 4096, H, mode=1) == {"peer_two_shot": 0, "switch": 0}


def test_clearing_device_error_bits_runs_the_reset_hooks(monkeypatch):
    """A kernel that gave up a wait may leave state behind (the stream-K GEMM's
    raised hand-off flags); reading and clearing non-zero error bits runs the
    registered resets, and the stream-K workspace's reset is one of them."""
    from kavor_b200 import _kernels, _lib

    assert _kernels.GEMM_WORKSPACE.reset in _lib._ON_CLEARED_ERROR
    seen = []
    monkeypatch.setattr(_lib, "_ON_CLEARED_ERROR", [seen.append])
    word = {"bits": 0}

    def fake_call(name, *args):
        assert name == "kvb_device_error"
        args[0]._obj.value = word["bits"]

    monkeypatch.setattr(_lib, "call", fake_call)
    assert _lib.device_error(clear=True) == 0 and seen == []
    word["bits"] = 4
    assert _lib.device_error(clear=False) == 4 and seen == []  # read only: nothing is reset
    assert _lib.device_error(clear=True) == 4 and seen == [4]


def test_every_entry_point_has_an_integration_entry():
    """Each declared entry point appears in the integration guide (its reference
    call site or its use), so the guide covers the whole boundary."""
    guide = (ROOT / "INTEGRATION.md").read_text()
    assert sorted(n for n in _declared() if n not in guide) == []
