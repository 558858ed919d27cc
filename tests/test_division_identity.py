"""The division the WARM quantizer relies on, checked on the CPU.

The reference divides fp16 tensors (`tensor / scale`, `diff / 255`,
`min_val / scale`; tierkv_policy.py:25-34): PyTorch evaluates x / s in fp32
and rounds to fp16.  The CUDA kernels (tkv_quant.cu) compute
fp16(x * fp32(1/s)) instead, which agrees for every fp16 x and s > 0 whenever
|x / s| >= 2^-14 (the argument is in tkv_quant.cu beside div_by); below that
the callers only round the quotient to an integer.  numpy's float32 multiply
and divide and its float32 -> float16 cast are IEEE round-to-nearest-even, as
the GPU instructions are, so this test pins the identity the kernels use.
All finite fp16 x against a sample of scales that includes the extremes; the
full x by s product (about 10^9 pairs) was also run once outside the suite.
"""

import numpy as np

rng = np.random.default_rng(20240611)

ALL_X = np.arange(0, 0x10000, dtype=np.uint32).astype(np.uint16).view(np.float16)
ALL_X = ALL_X[np.isfinite(ALL_X)].astype(np.float32)

_EXTREME_S = np.array([0x0001, 0x0002, 0x0003, 0x03FF, 0x0400, 0x0401, 0x3BFF, 0x3C00,
                       0x3C01, 0x5BF8, 0x7BFF], dtype=np.uint16)  # incl. 255 = 0x5BF8


def _scales():
    sample = rng.integers(1, 0x7C00, size=400).astype(np.uint16)
    return np.concatenate([_EXTREME_S, sample]).view(np.float16).astype(np.float32)


def test_reciprocal_multiply_rounds_like_the_division():
    with np.errstate(over="ignore"):
        for s in _scales():
            s = np.float32(s)
            r = np.float32(1.0) / s
            fast = (ALL_X * r).astype(np.float16)
            exact = (ALL_X / s).astype(np.float16)
            normal = np.abs(ALL_X / s) >= np.float32(2.0 ** -14)
            bad = normal & (fast.view(np.uint16) != exact.view(np.uint16))
            assert not bad.any(), (float(s), ALL_X[bad][:4])
            # subnormal quotients: the integer they round to, sign included
            tiny = ~normal
            fr = np.rint(fast[tiny].astype(np.float32))
            er = np.rint(exact[tiny].astype(np.float32))
            assert np.array_equal(fr.view(np.uint32), er.view(np.uint32)), float(s)


def test_scale_of_a_row_uses_the_constant_reciprocal_of_255():
    # scale = fp16(diff / 255) for every finite fp16 diff >= 0
    diff = ALL_X[ALL_X >= 0]
    inv255 = np.float32(1.0) / np.float32(255.0)
    fast = (diff * inv255).astype(np.float16)
    exact = (diff / np.float32(255.0)).astype(np.float16)
    assert np.array_equal(fast.view(np.uint16), exact.view(np.uint16))
