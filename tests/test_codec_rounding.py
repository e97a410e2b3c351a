"""The bulk encode kernel's quotient rounding without a division per value
(code_nibble_rcp in chronoquant_mlx_b200/csrc/cq_encode.cuh), restated in
float32 NumPy and checked against the reference rule it replaces: the
quotient delta / scale rounded to the token dtype, then half to even
(codec.py:48-51), for fp16 and bf16 operands.

The method: q' = delta * r with r = 1/scale correctly rounded; m = floor(q')
+ 1/2; h = half a dtype ulp at m; the code is rint(m) when lo = m - h <=
delta / scale <= hi = m + h (decided from the exact signs of delta - lo *
scale and delta - hi * scale, an FMA on the device, float64 here where the
products are exact) and rint(q') otherwise.  A scale whose reciprocal
overflows float32 (bf16 below 2^-126) is scaled by 2^64 with the residuals
first.  Half the samples are built to land near half-integers, where the
dtype rounding decides the code."""

import numpy as np

from oracle import cq_oracle as O


def _f32(x):
    return np.asarray(x, dtype=np.float32)


def method(dv, scale, dtype):
    dv, scale = _f32(dv), _f32(scale)
    with np.errstate(over="ignore", divide="ignore", invalid="ignore"):
        r = np.float32(1.0) / scale
        big = ~np.isfinite(r)
        up = np.where(big, np.float32(2.0 ** 64), np.float32(1.0)).astype(np.float32)
        dv = (dv * up).astype(np.float32)
        scale = (scale * up).astype(np.float32)
        r = (np.float32(1.0) / scale).astype(np.float32)
        q = (dv * r).astype(np.float32)
        m = (np.floor(q) + np.float32(0.5)).astype(np.float32)
        fb = 8 if dtype == "bf16" else 11
        h = ((m.view(np.int32) & np.int32(0x7F800000)) - np.int32(fb << 23)).view(np.float32)
        lo, hi = (m - h).astype(np.float32), (m + h).astype(np.float32)
        d64, s64 = dv.astype(np.float64), scale.astype(np.float64)
        on_half = (d64 - lo.astype(np.float64) * s64 >= 0) & (d64 - hi.astype(np.float64) * s64 <= 0)
        return np.where(on_half, np.rint(m), np.rint(q))


def reference(dv, scale, dtype):
    with np.errstate(over="ignore", divide="ignore", invalid="ignore"):
        qd = np.asarray(dv, np.float64) / np.asarray(scale, np.float64)
        qr = qd.astype(np.float16).astype(np.float64) if dtype == "f16" else O.round_bf16(qd.astype(np.float32))
        return np.rint(qr)


def samples(dtype, n, seed):
    rng = np.random.default_rng(seed)
    if dtype == "f16":
        scale = rng.integers(1, 0x7BFF, size=n).astype(np.uint16).view(np.float16).astype(np.float64)
        cast = lambda x: np.asarray(x, np.float64).astype(np.float16).astype(np.float64)
        fb = 11
    else:
        bits = rng.integers(1, 0x7F7F, size=n).astype(np.uint32) << np.uint32(16)
        scale = bits.view(np.float32).astype(np.float64)
        cast = lambda x: O.round_bf16(np.asarray(x, np.float32)).astype(np.float64)
        fb = 8
    t = rng.uniform(-8.0, 8.0, size=n)
    near = rng.random(n) < 0.5
    k = rng.integers(-8, 7, size=n) + 0.5
    h = 2.0 ** (np.floor(np.log2(np.abs(k))) - fb)
    t = np.where(near, k + rng.integers(-1, 2, size=n) * h + rng.uniform(-1e-6, 1e-6, size=n), t)
    with np.errstate(over="ignore"):
        dv = cast(t * scale)
    ok = np.isfinite(dv)
    return dv[ok], scale[ok]


def test_reciprocal_rounding_matches_dtype_division_f16():
    dv, scale = samples("f16", 2_000_000, 1)
    assert np.array_equal(method(dv, scale, "f16"), reference(dv, scale, "f16"))


def test_reciprocal_rounding_matches_dtype_division_bf16():
    dv, scale = samples("bf16", 2_000_000, 2)
    assert np.array_equal(method(dv, scale, "bf16"), reference(dv, scale, "bf16"))


def test_samples_reach_the_rounding_intervals():
    """The near-tie samples do land on half-integers after dtype rounding,
    and some of them only through the dtype rounding (the quotient itself is
    not a half-integer)."""
    for dtype in ("f16", "bf16"):
        dv, scale = samples(dtype, 200_000, 3)
        qd = dv / scale
        qr = qd.astype(np.float16).astype(np.float64) if dtype == "f16" else O.round_bf16(qd.astype(np.float32))
        landed = (qr - np.floor(qr)) == 0.5
        assert landed.sum() > 1000
        assert (landed & ((qd - np.floor(qd)) != 0.5)).sum() > 100
