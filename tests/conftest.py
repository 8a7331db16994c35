"""Shared pytest configuration.

``-m gpu`` tests need a B200 and the built ``kavor_b200/libkavor_b200.so``;
``-m "not gpu"`` tests run on any CPU (oracle vs golden fixtures, host-side
scheduling and metadata, library exports, gloo multi-rank logic).
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built kernel library")


@pytest.fixture(autouse=True)
def small_block_size(monkeypatch):
    """Scheduler/BlockManager unit tests use 4-token blocks like the reference's
    own suite (tests/conftest.py there); GPU tests set their own sizes."""
    from kavor_b200.engine.sequence import Sequence

    monkeypatch.setattr(Sequence, "block_size", 4)


@pytest.fixture
def make_seq():
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    def _make(token_ids, *, temperature=1.0, max_tokens=64, ignore_eos=False):
        return Sequence(list(token_ids), SamplingParams(temperature=temperature, max_tokens=max_tokens,
                                                        ignore_eos=ignore_eos))

    return _make


@pytest.fixture
def make_config():
    from types import SimpleNamespace

    def _make(**overrides):
        values = dict(max_num_seqs=8, max_num_batched_tokens=256, eos=0, kvcache_block_size=4,
                      num_kvcache_blocks=64)
        values.update(overrides)
        return SimpleNamespace(**values)

    return _make


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)
