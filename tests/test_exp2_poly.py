"""Error bound of the FMA-pipe exp2 used for part of the softmax (sm100_primitives.cuh).

The device function is restated step for step in float32 numpy with the coefficients read
from the header, and compared with exp2 in float64: relative error <= 1.1e-4 on [-125, 8]
(the softmax feeds exponents <= 8), exact zeros at and below -127 (fully masked rows keep a
zero row sum), tiny positive values in between.
"""
import os
import re

import numpy as np

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "loopfuse_b200",
                   "csrc", "sm100_primitives.cuh")


def coeffs():
    text = open(HDR).read()
    return [np.float32(float(re.search(rf"kExp2C{i} = ([0-9.e-]+)f;", text).group(1))) for i in (1, 2, 3)]


def emulate(t):
    c1, c2, c3 = coeffs()
    t = np.maximum(t.astype(np.float32), np.float32(-127))
    magic = np.float32(12582912.0)
    y = (t + magic).astype(np.float32)
    jf = (y - magic).astype(np.float32)
    f = (t - jf).astype(np.float32)
    p = ((c3 * f + c2) * f + c1) * f + np.float32(1)
    return (p.view(np.int32) + (y.view(np.int32) << 23)).view(np.float32)


def test_relative_error_bound():
    t = np.linspace(-125, 8, 1_000_001).astype(np.float32)
    r = emulate(t)
    ref = np.exp2(t.astype(np.float64))
    assert np.max(np.abs(r / ref - 1)) <= 1.1e-4


def test_masked_inputs_give_zero():
    t = np.array([-np.inf, -1e30, -300, -127.0, -127.0], dtype=np.float32)
    assert np.all(emulate(t) == 0)
    mid = emulate(np.linspace(-126.99, -125, 1001).astype(np.float32))
    assert np.all(mid >= 0) and np.all(mid < 3e-38)
