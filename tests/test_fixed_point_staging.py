"""The activation staging used by the one-row INT4 GEMV (w4_gemv_mma.cu, 32-k
halves) and the INT8 per-channel GEMV's decode path (dense_gemv.cu, 8-row
chunks), restated in numpy: x = 2^(E-21) q with E the exponent of the group's
largest |x|, q = round(x 2^(21-E)) = 65536 hi + 256 mid + lo in signed bytes.
The kernels then reduce the bytes exactly in int32, so the only approximation
is this staging; these CPU tests pin its bounds (|q| <= 2^22, hi, mid and lo
fit int8, and the reconstruction error is at most 2^-22 of the group's largest
|x|, or 2^-122 in absolute terms for groups whose largest |x| is below 2^-100,
where the exponent is clamped).

They also show why 24 bits: with one outlier of 100..1000 per group, a
16-bit staging misses the 2e-3 + 1e-2 |y| bar on columns whose sum nearly
cancels, and the 24-bit one does not."""
import numpy as np
import pytest


def split_bytes(q):
    lo = ((q + 128) & 255) - 128
    r = (q - lo) >> 8
    mid = ((r + 128) & 255) - 128
    hi = (r - mid) >> 8
    return hi, mid, lo


def stage(x, bits=24):
    """Per-group staging of a float32 group like the kernels (bits = 24), or
    the earlier 16-bit form (bits = 16) for comparison."""
    x = np.asarray(x, np.float32)
    m = np.float32(np.max(np.abs(x)))
    E = max(int((m.view(np.int32) >> 23)) - 127, -100)
    f = bits - 3
    inv = np.float32(2.0) ** np.float32(f - E)
    q = np.rint(x * inv).astype(np.int64)  # round half to even, like __float2int_rn
    return q, np.float64(2.0) ** (E - f), m


@pytest.mark.parametrize("n", [8, 32])
def test_bounds_random(n):
    rng = np.random.default_rng(n)
    for scale in (1e-32, 1e-6, 1.0, 3.0e4, 1e30):
        for _ in range(200):
            x = (rng.standard_normal(n) * scale).astype(np.float32)
            q, s, m = stage(x)
            hi, mid, lo = split_bytes(q)
            assert np.all(np.abs(q) <= 2 ** 22)
            for b in (hi, mid, lo):
                assert np.all((b >= -128) & (b <= 127))
            assert np.all(65536 * hi + 256 * mid + lo == q)
            err = np.abs(q * s - x.astype(np.float64))
            assert np.all(err <= max(2.0 ** -22 * float(m) * (1 + 1e-6), 2.0 ** -122))


def test_edge_groups():
    for x in ([0.0] * 8, [1.0] + [0.0] * 7, [-1.0] * 8, [np.float32(1.999999)] * 8,
              [np.float32(2.0 ** -126)] * 8, [np.float32(65504.0), -1e-3] + [0.0] * 6,
              [np.float32(-3.0e38)] + [1.0] * 7):
        q, s, m = stage(x)
        hi, mid, lo = split_bytes(q)
        assert np.all(np.abs(q) <= 2 ** 22)
        assert np.all(65536 * hi + 256 * mid + lo == q)
        err = np.abs(q * s - np.asarray(x, np.float64))
        assert np.all(err <= max(2.0 ** -22 * float(m), 2.0 ** -122))


def test_int32_partials_cannot_overflow():
    """The largest partial sums the kernels form before converting to float:
    INT4 GEMV, per 32-k half and column, 256 D_hi + D_mid - (8 + zero) S_hm;
    INT8 GEMV, per 8-row chunk and column, 256 hi_sum + mid_sum."""
    hi_max, mid_max, r_max = 64, 128, 2 ** 14 + 1
    int4_term = 256 * (32 * 15 * hi_max) + 32 * 15 * mid_max + 15 * 32 * r_max
    int8_term = 256 * (8 * 128 * hi_max) + 8 * 128 * mid_max
    assert int4_term < 2 ** 31 and int8_term < 2 ** 31
    assert int4_term < 2 ** 25  # within two bits of float's 24-bit mantissa: one rounding


@pytest.mark.parametrize("amp", [100.0, 1000.0])
def test_outliers_need_24_bits(amp):
    """K = 1024 activations ~ N(0,1) with one outlier of +-amp per 32 k,
    against 512 random weight columns: the 16-bit staging misses the bar on
    some columns, the 24-bit staging on none."""
    rng = np.random.default_rng(int(amp))
    K, N = 1024, 512
    x = rng.standard_normal(K).astype(np.float32)
    idx = np.arange(0, K, 32) + rng.integers(0, 32, K // 32)
    x[idx] = (amp * np.sign(rng.standard_normal(K // 32))).astype(np.float32)
    W = rng.integers(-8, 8, (K, N)).astype(np.float64) * 0.004
    want = x.astype(np.float64) @ W

    def staged(bits):
        out = np.empty(K)
        for h in range(0, K, 32):
            q, s, _ = stage(x[h:h + 32], bits)
            out[h:h + 32] = q * s
        return out @ W

    def misses(y):
        return int((np.abs(y - want) > 2e-3 + 1e-2 * np.abs(want)).sum())

    assert misses(staged(24)) == 0
    assert misses(staged(16)) > 0
