"""The FMA-pipe 2^x of the prefill softmax (exp2_fma in prefill_attn.cu):
the cubic read from the source, evaluated in float32 with the same exponent
split, stays within 1e-4 relative of 2^x over the range the softmax uses
(x in [-126, 0]) and is exactly 0 below it."""
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "kavor_b200" / "csrc" / "prefill_attn.cu"


def _coeffs():
    m = re.search(r"fmaf\(fmaf\(fmaf\(([0-9.e+-]+)f, f, ([0-9.e+-]+)f\), f, ([0-9.e+-]+)f\), f, 1\.0f\)",
                  SRC.read_text())
    assert m, "exp2_fma polynomial not found"
    return [np.float32(v) for v in m.groups()]


def _exp2_fma(x: np.ndarray) -> np.ndarray:
    c3, c2, c1 = _coeffs()
    x = x.astype(np.float32)
    xc = np.maximum(x, np.float32(-127))  # the kernel returns 0 before computing below -126
    i = np.floor(xc)
    f = (xc - i).astype(np.float32)
    p = ((c3 * f + c2) * f + c1) * f + np.float32(1.0)
    bits = p.astype(np.float32).view(np.int32) + (i.astype(np.int32) << 23)
    out = bits.view(np.float32)
    return np.where(x < -126, np.float32(0), out)


def test_exp2_fma_relative_error():
    x = np.linspace(-126, 0, 2_000_001, dtype=np.float64)
    got = _exp2_fma(x).astype(np.float64)
    ref = np.exp2(x)
    assert np.max(np.abs(got / ref - 1)) < 1e-4
    assert _exp2_fma(np.array([-126.5, -1e30, -np.inf]))[:].tolist() == [0.0, 0.0, 0.0]
    assert _exp2_fma(np.array([0.0]))[0] == 1.0
