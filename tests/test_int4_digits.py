"""The INT4 integer path stages x 2^s as three signed base-128 digits (mirror of the split in stage_x, integer path):
t = v + 64 (1 + 128 + 128^2), d0 = (t & 127) - 64, d1 = ((t >> 7) & 127) - 64, d2 = (t >> 14) - 64. Checked for every
integer v the staging can produce (|v| <= 2^20): exact reconstruction and every digit inside int8."""
import numpy as np


def test_digit_split_is_exact_for_every_staged_integer():
    v = np.arange(-(1 << 20), (1 << 20) + 1, dtype=np.int64)
    t = v + 1056832
    assert t.min() >= 0
    d0 = (t & 127) - 64
    d1 = ((t >> 7) & 127) - 64
    d2 = (t >> 14) - 64
    assert np.array_equal(d0 + 128 * d1 + 16384 * d2, v)
    for d in (d0, d1, d2):
        assert d.min() >= -128 and d.max() <= 127
    assert d0.min() == -64 and d0.max() == 63 and d2.max() == 64


def test_group_sums_fit_int32_and_the_fold_is_exact_in_int32():
    # per 128-group: |D_d| <= 128 * 15 * 64 (u8 nibbles times digits), |S_d| <= 128 * 64
    assert 128 * 15 * 64 < 2 ** 31 and 128 * 64 * 8 < 2 ** 31


def _f32(v):
    return np.float32(v)


def _fma(a, b, c):
    """fmaf: one rounding of a * b + c (exact in float64 for these magnitudes)."""
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def test_split_nibble_fold_matches_the_exact_group_sum():
    """Mirror of the TMA kernel's integer INT4 step: per 128-group and row, chain L = low nibbles (even k) against
    the even-k digits, chain H = high nibbles kept as 16 n (odd k) against the odd-k digits; lane c = 0 folds digits
    0, 1 and lane c = 1 digit 2 as (16 L + H) 128^d / 16 - C with C = 8 sum 128^d S_d staged per group. Every
    intermediate is an exact float and the two lanes add up to sum_d 128^d (D_d - 8 S_d) to float rounding."""
    rng = np.random.default_rng(3)
    for trial in range(200):
        if trial == 0:
            q = np.full(128, 15)
            dg = np.full((3, 128), 64)
            dg[:2] = 63
        elif trial == 1:
            q = np.full(128, 15)
            dg = np.full((3, 128), -64)
        else:
            q = rng.integers(0, 16, 128)
            dg = np.stack([rng.integers(-64, 64, 128), rng.integers(-64, 64, 128), rng.integers(-64, 65, 128)])
        even, odd = slice(0, None, 2), slice(1, None, 2)
        L = [int((q[even] * dg[d][even]).sum()) for d in range(3)]
        H = [int((16 * q[odd] * dg[d][odd]).sum()) for d in range(3)]
        S = [int(dg[d].sum()) for d in range(3)]
        exact = sum(128 ** d * (int((q * dg[d]).sum()) - 8 * S[d]) for d in range(3))
        for d in range(3):
            assert abs(16 * L[d] + H[d]) < 2 ** 21                     # exact as a float
        c0 = _f32(8.0 * (_f32(S[0]) + _f32(128.0 * S[1])))            # staged offsets, exact
        c1 = _f32(131072.0 * S[2])
        assert float(c0) == 8 * (S[0] + 128 * S[1]) and float(c1) == 131072 * S[2]
        lane0 = _fma(_f32(16 * L[0] + H[0]), 0.0625, _fma(_f32(16 * L[1] + H[1]), 8.0, -c0))
        lane1 = _fma(_f32(16 * L[2] + H[2]), 1024.0, _fma(_f32(0), 0.0, -c1))
        got = float(np.float32(lane0 + lane1))
        assert abs(got - exact) <= 2.0 ** -22 * max(abs(exact), 2.0 ** 24 * 2.0 ** -4), (trial, got, exact)
