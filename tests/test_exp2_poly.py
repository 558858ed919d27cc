"""The FMA-pipe exp2 of the prefill kernels (ex2_fma in csrc/tkv_ptx.cuh),
replayed step for step in numpy float32: its relative error against exp2
stays below the bound its comment states, over the whole input range the
kernels feed it (logits minus a running max: x <= 0), and inputs at or below
the clamp give values below 2^-124 that never turn negative or non-finite."""

import os
import re

import numpy as np

HEADER = os.path.join(os.path.dirname(__file__), "..", "paged_tierkv_b200", "csrc", "tkv_ptx.cuh")


def _coefficients():
    src = open(HEADER).read()
    c = [float(re.search(rf"kExp2Poly{i} = ([0-9.e+-]+)f;", src).group(1)) for i in range(5)]
    return np.array(c, dtype=np.float32)


def ex2_fma(x):
    c = _coefficients()
    x = np.maximum(np.asarray(x, np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic).astype(np.float32)).astype(np.float32)
    p = c[4]
    for k in (3, 2, 1, 0):  # fmaf: one rounding per step
        p = (p.astype(np.float64) * f + c[k]).astype(np.float32)
    bits = p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_relative_error_bound():
    rng = np.random.default_rng(3)
    x = np.concatenate([np.linspace(-125.0, 0.0, 2_000_001, dtype=np.float32),
                        -rng.exponential(4.0, 1_000_000).astype(np.float32)])
    x = x[x >= -125.0]
    y = ex2_fma(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(y / ref - 1.0)) < 3e-6


def test_clamped_inputs_stay_tiny_and_positive():
    x = np.array([-np.inf, -1e30, -500.0, -126.0, -125.6], dtype=np.float32)
    y = ex2_fma(x)
    assert np.all(np.isfinite(y)) and np.all(y >= 0) and np.all(y < 2.0 ** -124)
