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
