"""The activation staging used by the one-row INT4 GEMV (w4_gemv_mma.cu, 32-k
halves) and the INT8 per-channel GEMV's decode path (dense_gemv.cu, 8-row
chunks), restated in numpy: x = 2^(E-13) q with E the exponent of the group's
largest |x|, q = round(x 2^(13-E)) = 256 hi + lo in signed bytes.  The kernels
then reduce the bytes exactly in int32, so the only approximation is this
staging; these CPU tests pin its bounds (|q| <= 2^14, hi and lo fit int8, and
the reconstruction error is at most 2^-14 of the group's largest |x|, or 2^-114
in absolute terms for groups whose largest |x| is below 2^-100, where the
exponent is clamped)."""
import numpy as np
import pytest


def stage(x):
    """Per-group staging of a float32 group as (hi, lo, scale) like the kernels."""
    x = np.asarray(x, np.float32)
    m = np.float32(np.max(np.abs(x)))
    E = max(int((m.view(np.int32) >> 23)) - 127, -100)
    inv = np.float32(2.0) ** np.float32(13 - E)
    q = np.rint(x * inv).astype(np.int64)  # round half to even, like __float2int_rn
    lo = ((q + 128) & 255) - 128
    hi = (q - lo) >> 8
    return hi, lo, np.float64(2.0) ** (E - 13), q, m


@pytest.mark.parametrize("n", [8, 32])
def test_bounds_random(n):
    rng = np.random.default_rng(n)
    for scale in (1e-30, 1e-6, 1.0, 3.0e4, 1e30):
        for _ in range(200):
            x = (rng.standard_normal(n) * scale).astype(np.float32)
            hi, lo, s, q, m = stage(x)
            assert np.all(np.abs(q) <= 2 ** 14)
            assert np.all((hi >= -128) & (hi <= 127)) and np.all((lo >= -128) & (lo <= 127))
            assert np.all(256 * hi + lo == q)
            err = np.abs((256 * hi + lo) * s - x.astype(np.float64))
            assert np.all(err <= max(2.0 ** -14 * float(m) * (1 + 1e-6), 2.0 ** -114))


def test_edge_groups():
    for x in ([0.0] * 8, [1.0] + [0.0] * 7, [-1.0] * 8, [np.float32(1.999999)] * 8,
              [np.float32(2.0 ** -126)] * 8, [np.float32(65504.0), -1e-3] + [0.0] * 6):
        hi, lo, s, q, m = stage(x)
        assert np.all(np.abs(q) <= 2 ** 14)
        err = np.abs((256 * hi + lo) * s - np.asarray(x, np.float64))
        assert np.all(err <= max(2.0 ** -14 * float(m), 2.0 ** -114))
