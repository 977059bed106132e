"""The FMA-pipe 2^x of the prefill softmax (csrc/prefill.cu exp2_poly_pair),
re-evaluated on the CPU in FP32 exactly as the device does: Cody-Waite split
with the 1.5*2^23 shifter, degree-4 polynomial, exponent added as an integer."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(__file__)), "gpullama3.java_b200", "csrc",
                   "prefill.cu")


def coefficients():
    text = open(SRC).read()
    vals = dict(re.findall(r"(kE2C\d) = (0x[0-9a-fA-Fp.+-]+)f", text))
    return [np.float32(float.fromhex(vals[f"kE2C{i}"])) for i in range(5)]


def exp2_poly(x):
    c = coefficients()
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-126.0))
    shift = np.float32(12582912.0)
    t = (x + shift).astype(np.float32)
    n = (t - shift).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = c[4]
    for ci in (c[3], c[2], c[1], c[0]):
        p = (p * f + ci).astype(np.float32)  # separate rounding bounds the FMA error too
    bits = p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.int32).view(np.float32)


def test_relative_error_over_softmax_range():
    x = np.linspace(-100.0, 8.0, 2_000_001, dtype=np.float32)
    got = exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 5e-6, rel.max()


def test_reduced_argument_range():
    f = np.linspace(-0.5, 0.5, 100_001, dtype=np.float32)
    rel = np.abs(exp2_poly(f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)
    assert rel.max() < 5e-6


def test_masked_scores_vanish_in_fp16():
    y = exp2_poly(np.array([-np.inf, -1000.0, -126.0], dtype=np.float32))
    assert np.all(y >= 0) and np.all(y < 1e-37)
    assert np.all(y.astype(np.float16) == 0)
