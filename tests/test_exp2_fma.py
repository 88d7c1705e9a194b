"""The attention softmax computes one exponent pair in four on the FMA pipe (exp2_fma_x2 in
csrc/attention.cu): n = round(x) through the 1.5 * 2^23 shift, a degree-4 polynomial for
2^(x - n) on [-1/2, 1/2], n added to the exponent field, 0 for arguments below -126.  This test
reads the polynomial's coefficients from the kernel source (so the two cannot drift apart) and
replays the construction in float32 on the CPU: relative error below 3e-6 over the range the
softmax uses, exact zeros for masked keys, no negative or NaN results."""

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "rldx-1_b200" / "csrc" / "attention.cu"


def coefficients():
    body = SRC.read_text()
    fn = body[body.index("exp2_fma_x2(float2 x)"):]
    # the Horner chain only: it starts from the highest coefficient, then adds the others in turn
    fn = fn[fn.index("float2 p = "):fn.index("return make_float2")]
    lits = re.findall(r"make_float2\(([0-9.]+)f, \1f\)", fn)
    assert len(lits) == 5, lits
    return [np.float32(v) for v in lits]


def exp2_fma(x):
    c = coefficients()
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        t = (x + np.float32(12582912.0)).astype(np.float32)
        n = (t - np.float32(12582912.0)).astype(np.float32)
        f = (x - n).astype(np.float32)
        p = np.full_like(x, c[0])
        for k in c[1:]:
            p = (p * f + k).astype(np.float32)
        bits = (p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
        r = bits.astype(np.uint32).view(np.int32).view(np.float32)
    return np.where(x >= -126.0, r, np.float32(0.0))


def test_relative_error_over_the_softmax_range():
    # arguments of the softmax exponentials: scores minus a lazily moved reference max, so at
    # most 2^8 above it (x <= 8), down to where the result no longer matters
    x = np.linspace(-125.0, 9.0, 1_000_001, dtype=np.float32)
    got = exp2_fma(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got / ref - 1.0)) < 3e-6


def test_masked_and_tiny_arguments_give_zero():
    x = np.array([-np.inf, -1e30, -200.0, -127.0, -126.5], dtype=np.float32)
    assert np.all(exp2_fma(x) == 0.0)


def test_no_negative_or_nan_results():
    x = np.linspace(-126.0, 9.0, 200_001, dtype=np.float32)
    r = exp2_fma(x)
    assert not np.any(np.isnan(r)) and np.all(r > 0.0)
