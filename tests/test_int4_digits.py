"""The INT4 integer path stages v = x 2^s (an integer, |v| < 2^30) as four signed base-256 digits (mirror of the split
in stage_x, integer path): t = v + 0x80808080 lies in [0, 2^32), its bytes b_d are the balanced digits offset by 128,
and b_d ^ 0x80 read as an int8 is d_d. Checked on the CPU: exact reconstruction and int8 digits for the integers the
staging produces, the byte transposes into the digit planes, the packed group sums, and the consumers' per-group fold."""
import numpy as np

OFFSET = 0x80808080


def split(v):
    """(digits [4, n] int64, t uint32) of integers v."""
    t = (v.astype(np.int64) + OFFSET) & 0xFFFFFFFF
    d = np.stack([((t >> (8 * k)) & 0xFF) ^ 0x80 for k in range(4)]).astype(np.int64)
    d = np.where(d >= 128, d - 256, d)                        # the byte as an int8
    return d, t


def test_digit_split_is_exact_for_every_staged_integer():
    lim = 1 << 30
    rng = np.random.default_rng(0)
    v = np.concatenate([np.arange(-lim + 1, -lim + 300001), np.arange(lim - 300000, lim),
                        np.arange(-300000, 300001), rng.integers(-lim + 1, lim, 4_000_000)]).astype(np.int64)
    d, t = split(v)
    assert ((v + OFFSET) >= 0).all() and ((v + OFFSET) < 2 ** 32).all()   # the uint32 add never wraps
    assert np.array_equal(d[0] + 256 * d[1] + 65536 * d[2] + 16777216 * d[3], v)
    assert d.min() >= -128 and d.max() <= 127
    assert d[3].min() >= -64 and d[3].max() <= 64


def test_staged_integers_are_exact_for_elements_within_2_22_of_max():
    """v = x 2^s with max|x| 2^s in [2^29, 2^30): every bf16 x within 2^22 of max|x| is an integer after scaling."""
    bits = np.arange(0, 0x7F80, dtype=np.uint32)               # every finite positive bf16
    x = (bits << 16).view(np.float32).astype(np.float64)
    for ex in (-20, 0, 7, 60):
        s = 29 - ex
        keep = (x >= 2.0 ** (ex - 22)) & (x < 2.0 ** (ex + 1))
        v = x[keep] * 2.0 ** s
        assert np.array_equal(v, np.round(v)) and v.max() < 2 ** 30


def byte_perm(x, y, sel):
    """__byte_perm(x, y, sel): byte n of the result is byte (sel >> 4n) & 7 of the 8 bytes {y, x} (x low)."""
    src = [(x >> (8 * k)) & 0xFF for k in range(4)] + [(y >> (8 * k)) & 0xFF for k in range(4)]
    return sum(src[(sel >> (4 * n)) & 7] << (8 * n) for n in range(4))


def test_byte_transposes_build_the_digit_planes():
    """The kernel's 4 x 4 transposes: element words t0..t7 -> plane d words (x0, x2, x4, x6) and (x1, x3, x5, x7)."""
    rng = np.random.default_rng(5)
    for _ in range(200):
        v = rng.integers(-(1 << 30) + 1, 1 << 30, 8)
        d, t = split(v)
        t = [int(w) for w in t]
        for h in range(2):
            a, b = byte_perm(t[h], t[h + 2], 0x5140), byte_perm(t[h], t[h + 2], 0x7362)
            c, e = byte_perm(t[h + 4], t[h + 6], 0x5140), byte_perm(t[h + 4], t[h + 6], 0x7362)
            words = [byte_perm(a, c, 0x5410), byte_perm(a, c, 0x7632), byte_perm(b, e, 0x5410),
                     byte_perm(b, e, 0x7632)]
            for k in range(4):
                w = words[k] ^ 0x80808080
                got = [((w >> (8 * n)) & 0xFF) for n in range(4)]
                got = [g - 256 if g >= 128 else g for g in got]
                assert got == [int(d[k][h + 2 * n]) for n in range(4)]


def test_packed_group_sums_decode_exactly():
    """Digit sums travel two per word (S_a + 65536 S_b) through the 16-lane reduction: |S| <= 16384 decodes exactly."""
    rng = np.random.default_rng(9)
    for _ in range(2000):
        sa = rng.integers(-1024, 1025, 16)
        sb = rng.integers(-1024, 1025, 16)
        packed = int(np.sum(sa + 65536 * sb))
        assert abs(packed) < 2 ** 31
        lo = (packed & 0xFFFF)
        lo = lo - 65536 if lo >= 32768 else lo
        assert lo == sa.sum() and (packed - lo) >> 16 == sb.sum()


def _f32(v):
    return np.float32(v)


def _fma(a, b, c):
    """fmaf: one rounding of a * b + c (exact in float64 for these magnitudes)."""
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def test_split_nibble_fold_matches_the_exact_group_sum():
    """Mirror of the TMA kernel's integer INT4 step: per 128-group and row, chain L = low nibbles (even k) against
    the even-k digits, chain H = high nibbles kept as 16 n (odd k) against the odd-k digits; with t_d = 16 L_d + H_d,
    lane c = 0 folds digits 0, 1 as (t_0 + 256 t_1) / 16 - C_0 and lane c = 1 digits 2, 3 as (t_2 + 256 t_3) 4096 - C_1
    (the two digits merged in int32, one conversion each), C = 8 sum 256^d S_d staged per group. The two lanes add up
    to sum_d 256^d (D_d - 8 S_d) to float rounding."""
    rng = np.random.default_rng(3)
    for trial in range(300):
        if trial == 0:
            q = np.full(128, 15)
            dg = np.full((4, 128), 127)
            dg[3] = 64
        elif trial == 1:
            q = np.full(128, 15)
            dg = np.full((4, 128), -128)
            dg[3] = -64
        elif trial == 2:                                        # one outlier element, the rest small
            q = rng.integers(0, 16, 128)
            dg = np.zeros((4, 128), dtype=np.int64)
            dg[0] = rng.integers(-128, 128, 128)
            dg[3, 5] = 64
        else:
            q = rng.integers(0, 16, 128)
            dg = np.stack([rng.integers(-128, 128, 128), rng.integers(-128, 128, 128), rng.integers(-128, 128, 128),
                           rng.integers(-64, 65, 128)])
        even, odd = slice(0, None, 2), slice(1, None, 2)
        L = [int((q[even] * dg[d][even]).sum()) for d in range(4)]
        H = [int((16 * q[odd] * dg[d][odd]).sum()) for d in range(4)]
        S = [int(dg[d].sum()) for d in range(4)]
        exact = sum(256 ** d * (int((q * dg[d]).sum()) - 8 * S[d]) for d in range(4))
        t = [16 * L[d] + H[d] for d in range(4)]
        for d in range(4):
            assert abs(t[d]) < 2 ** 22
        m0, m1 = t[0] + 256 * t[1], t[2] + 256 * t[3]
        assert abs(m0) < 2 ** 31 and abs(m1) < 2 ** 31                  # the int32 merges do not overflow
        lo, hi = _f32(S[0] + 256 * S[1]), _f32(S[2] + 256 * S[3])
        c0, c1 = _f32(8.0 * lo), _f32(524288.0 * hi)                   # staged offsets, exact
        assert float(c0) == 8 * (S[0] + 256 * S[1]) and float(c1) == 524288 * (S[2] + 256 * S[3])
        lane0 = _fma(_f32(m0), 0.0625, -c0)
        lane1 = _fma(_f32(m1), 4096.0, -c1)
        got = float(np.float32(lane0 + lane1))
        # the conversions round relative to the merged integers, each fmaf and the add relative to their results
        l0, l1 = m0 / 16 - 8 * (S[0] + 256 * S[1]), m1 * 4096 - 524288 * (S[2] + 256 * S[3])
        bound = 2.0 ** -23 * (abs(m0) / 16 + abs(m1) * 4096 + abs(l0) + abs(l1) + abs(exact))
        assert abs(got - exact) <= bound, (trial, got, exact, bound)
