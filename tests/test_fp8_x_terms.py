"""The FP8 e4m3 path (TMA kernel, math 8) stages x as four e4m3 terms in two exponent tiers (mirror of stage_x, FP8
DEC 3): v = x 2^-e with max|x| 2^-e in [128, 256); hi0 = RN(v), lo0 = RN(v - hi0); r = v - hi0 - lo0;
hi1 = RN(2^16 r), lo1 = RN(2^16 r - hi1); the kernel sums hi0 + lo0 + 2^-16 (hi1 + lo1). Checked on the CPU for
every finite bf16 value: no term saturates, every residual is exact in fp32, x is reproduced exactly within 2^25 of
max|x| and to 2^-33 max|x| below that."""
import numpy as np
import torch


def e4m3_rn(v):
    """Round-to-nearest-even to e4m3 (what cvt.rn.satfinite.e4m3x2.f32 does for |v| <= 448), as float32."""
    return torch.from_numpy(v).to(torch.float8_e4m3fn).to(torch.float32).numpy()


def four_terms(v):
    v = v.astype(np.float32)
    hi0 = e4m3_rn(v)
    r = (v - hi0).astype(np.float32)
    lo0 = e4m3_rn(r)
    r = ((r - lo0) * np.float32(65536.0)).astype(np.float32)
    hi1 = e4m3_rn(r)
    lo1 = e4m3_rn((r - hi1).astype(np.float32))
    return hi0, lo0, hi1, lo1


def test_four_term_split_is_exact_within_2_25_of_max():
    bits = np.arange(0, 0x7F80, dtype=np.uint32)                  # every finite positive bf16
    x = (bits << 16).view(np.float32)
    x = np.concatenate([x, -x])
    for mx in (1.0, 3.0, 2000.0, 1e-20, 3e38):
        ex = int(np.floor(np.log2(mx)))
        e = ex - 7
        keep = np.abs(x.astype(np.float64)) <= mx
        xs = x[keep]
        v = (xs.astype(np.float64) * 2.0 ** -e).astype(np.float32)
        big = np.abs(xs.astype(np.float64)) >= mx * 2.0 ** -25
        assert np.array_equal(v[big].astype(np.float64), xs[big].astype(np.float64) * 2.0 ** -e)   # exact scaling
        hi0, lo0, hi1, lo1 = four_terms(v)
        for t in (hi0, lo0, hi1, lo1):
            assert np.isfinite(t).all() and np.abs(t).max() <= 448.0
        # residuals exact in fp32: recompute them in float64
        r1 = v.astype(np.float64) - hi0 - lo0
        assert np.abs(r1).max() <= 2.0 ** -10
        rec = (hi0.astype(np.float64) + lo0 + (hi1.astype(np.float64) + lo1) * 2.0 ** -16) * 2.0 ** e
        err = np.abs(rec - xs.astype(np.float64))
        assert err[big].max() == 0.0, mx
        assert err.max() <= mx * 2.0 ** -33, mx


def test_two_terms_alone_lose_bits_below_2_9_of_max():
    """Why tier 1 exists: hi0 + lo0 alone misses elements ~2^-10 of max|x| (an activation with a 1000x outlier)."""
    v = np.array([0.125 * (1 + 2.0 ** -7)], dtype=np.float32)     # 8 significant bits, 2^-10 of 128
    hi0, lo0, hi1, lo1 = four_terms(v)
    assert float(hi0[0] + lo0[0]) != float(v[0])
    assert float(hi0[0] + lo0[0] + (hi1[0] + lo1[0]) * 2.0 ** -16) == float(v[0])
