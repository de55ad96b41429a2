"""The attention's FMA-pipe exp2 (csrc/attention.cu ex2_poly) mirrored step for step in float32 numpy: the range
reduction with the 1.5 * 2^23 rounding constant, the degree-3 polynomial and the integer exponent add must give
2^x within 8e-5 relative over the whole softmax argument range, tiny non-negative values below -126, and ~0 for -inf."""
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "minimax-h3-2x-dgx-spark-tp2_b200" / "csrc" / "attention.cu"


def _coeffs():
    body = SRC.read_text().split("ex2_poly(float x) {", 1)[1].split("}", 1)[0]
    return [np.float32(float(v)) for v in re.findall(r"fmaf\([^;]*?([0-9]\.[0-9]+)f\)", body)] + \
        [np.float32(float(re.search(r"fmaf\(([0-9.]+)f, f", body).group(1)))]


def ex2_poly(x):
    c_round = np.float32(12582912.0)
    c2, c1, c0, c3 = _coeffs()          # source order: (c3 * f + c2), then c1, then c0
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    j = (x + c_round).astype(np.float32)
    f = (x - (j - c_round)).astype(np.float32)
    p = (c3 * f + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = p.view(np.int32) + (j.view(np.int32).astype(np.int64) << 23).astype(np.int64).astype(np.int32)
    return bits.astype(np.int32).view(np.float32)


def test_relative_error_over_the_softmax_range():
    x = np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32)
    got = ex2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 8e-5


def test_underflow_and_minus_infinity():
    x = np.array([-126.0, -130.0, -1e30, -np.inf], dtype=np.float32)
    got = ex2_poly(x)
    assert np.all(got >= 0) and np.all(got < 2e-38) and np.all(np.isfinite(got))
