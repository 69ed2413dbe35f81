"""The INT4 integer path stages x 2^s as four signed base-128 digits (mirror of the split in stage_x, integer path):
t = v + 64 (1 + 128 + 128^2 + 128^3), d_i = ((t >> 7 i) & 127) - 64 for i < 3, d3 = (t >> 21) - 64. Checked for the
integers the staging can produce (|v| <= 2^27): exact reconstruction and every digit inside int8."""
import numpy as np

OFFSET = 64 * (1 + 128 + 128 ** 2 + 128 ** 3)           # 135274560


def split(v):
    t = v + OFFSET
    return ((t & 127) - 64, ((t >> 7) & 127) - 64, ((t >> 14) & 127) - 64, (t >> 21) - 64), t


def test_digit_split_is_exact_for_every_staged_integer():
    lim = 1 << 27
    rng = np.random.default_rng(0)
    v = np.concatenate([np.arange(-lim, -lim + 300000), np.arange(lim - 300000, lim + 1),
                        np.arange(-300000, 300001), rng.integers(-lim, lim + 1, 4_000_000)]).astype(np.int64)
    (d0, d1, d2, d3), t = split(v)
    assert t.min() >= 0 and t.max() < 2 ** 31                  # the int32 offset add never overflows
    assert np.array_equal(d0 + 128 * d1 + 16384 * d2 + 2097152 * d3, v)
    for d in (d0, d1, d2, d3):
        assert d.min() >= -128 and d.max() <= 127
    assert d0.min() == -64 and d0.max() == 63 and d3.min() == -64 and d3.max() == 64


def test_staged_integers_are_exact_for_elements_within_2_19_of_max():
    """v = x 2^s with max|x| 2^s in [2^26, 2^27): every bf16 x within 2^19 of max|x| is an integer after scaling."""
    bits = np.arange(0, 0x7F80, dtype=np.uint32)               # every finite positive bf16
    x = (bits << 16).view(np.float32).astype(np.float64)
    for mx_exp in (-20, 0, 7, 60):
        ex = mx_exp
        s = 26 - ex
        keep = (x >= 2.0 ** (ex - 19)) & (x < 2.0 ** (ex + 1))
        v = x[keep] * 2.0 ** s
        assert np.array_equal(v, np.round(v)) and v.max() < 2 ** 27


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
    0, 1 and lane c = 1 digits 2, 3 as (16 L + H) 128^d / 16 - C with C = 8 sum 128^d S_d staged per group. Every
    product is an exact float and the two lanes add up to sum_d 128^d (D_d - 8 S_d) to float rounding."""
    rng = np.random.default_rng(3)
    for trial in range(300):
        if trial == 0:
            q = np.full(128, 15)
            dg = np.full((4, 128), 63)
            dg[3] = 64
        elif trial == 1:
            q = np.full(128, 15)
            dg = np.full((4, 128), -64)
        elif trial == 2:                                        # one outlier element, the rest small
            q = rng.integers(0, 16, 128)
            dg = np.zeros((4, 128), dtype=np.int64)
            dg[0] = rng.integers(-64, 64, 128)
            dg[3, 5] = 64
        else:
            q = rng.integers(0, 16, 128)
            dg = np.stack([rng.integers(-64, 64, 128), rng.integers(-64, 64, 128), rng.integers(-64, 64, 128),
                           rng.integers(-64, 65, 128)])
        even, odd = slice(0, None, 2), slice(1, None, 2)
        L = [int((q[even] * dg[d][even]).sum()) for d in range(4)]
        H = [int((16 * q[odd] * dg[d][odd]).sum()) for d in range(4)]
        S = [int(dg[d].sum()) for d in range(4)]
        exact = sum(128 ** d * (int((q * dg[d]).sum()) - 8 * S[d]) for d in range(4))
        for d in range(4):
            assert abs(16 * L[d] + H[d]) < 2 ** 21                     # exact as a float
        c0 = _f32(8.0 * (_f32(S[0]) + _f32(128.0 * S[1])))            # staged offsets, exact
        c1 = _f32(131072.0 * (_f32(S[2]) + _f32(128.0 * S[3])))
        assert float(c0) == 8 * (S[0] + 128 * S[1]) and float(c1) == 131072 * (S[2] + 128 * S[3])
        lane0 = _fma(_f32(16 * L[0] + H[0]), 0.0625, _fma(_f32(16 * L[1] + H[1]), 8.0, -c0))
        lane1 = _fma(_f32(16 * L[2] + H[2]), 1024.0, _fma(_f32(16 * L[3] + H[3]), 131072.0, -c1))
        got = float(np.float32(lane0 + lane1))
        # each fmaf rounds once relative to its own exact result, the add relative to the sum: the error is float
        # rounding of the lanes' exact partial values, not of the (larger) products that cancel inside an fmaf
        in0 = (16 * L[1] + H[1]) * 8 - 8 * (S[0] + 128 * S[1])
        in1 = (16 * L[3] + H[3]) * 131072 - 131072 * (S[2] + 128 * S[3])
        l0 = (16 * L[0] + H[0]) / 16 + in0
        l1 = (16 * L[2] + H[2]) * 1024 + in1
        bound = 2.0 ** -23 * (abs(in0) + abs(in1) + abs(l0) + abs(l1) + abs(exact))
        assert abs(got - exact) <= bound, (trial, got, exact, bound)
