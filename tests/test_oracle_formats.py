"""CPU: the oracle's number formats, pinned by the reference's known answers and, where the reference checkout is
present, by the reference's own compiled code (oracle/_ref/).

The known-answer checks restate src/tests/quant_host_selftest.cpp:9-46 against the oracle: e4m3 special codes,
round trip of every finite code, nearest code with ties to even by brute force, fp16 over all 65536 patterns, INT4
round-trip error <= s/2 with nibbles in 1..15, FP8 round-trip within one step."""
import subprocess

import numpy as np
import pytest

import oracle as O


def test_e4m3_known_answers():
    d = O.e4m3_decode(np.array([0x7E, 0x01, 0x38, 0xB8, 0x7F, 0xFF, 0x00, 0x80], dtype=np.uint8))
    assert d[0] == 448.0 and d[1] == 2.0 ** -9 and d[2] == 1.0 and d[3] == -1.0
    assert np.isnan(d[4]) and np.isnan(d[5]) and d[6] == 0.0 and d[7] == 0.0 and np.signbit(d[7])


def test_e4m3_every_finite_code_round_trips():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    back = O.e4m3_encode(O.e4m3_decode(codes))
    assert np.array_equal(back, codes)


def test_e4m3_nearest_code_ties_to_even_bruteforce():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-500, 500, 60000), rng.uniform(-0.5, 0.5, 30000) * 1e-3,
                        # exact midpoints between neighbouring codes
                        (O.e4m3_decode(np.arange(0, 126, dtype=np.uint8)) +
                         O.e4m3_decode(np.arange(1, 127, dtype=np.uint8))) / 2]).astype(np.float32)
    got = O.e4m3_encode(x)
    tab = O.e4m3_decode(np.arange(127, dtype=np.uint8)).astype(np.float64)
    a = np.minimum(np.abs(x.astype(np.float64)), 448.0)
    d = np.abs(a[:, None] - tab[None, :])
    best = d.min(axis=1, keepdims=True)
    cand = d == best
    # among equally near codes take the even one
    even = cand & (np.arange(127)[None, :] % 2 == 0)
    want = np.where(even.any(axis=1), even.argmax(axis=1), cand.argmax(axis=1))
    assert np.array_equal(got & 0x7F, want.astype(np.uint8))
    assert np.array_equal((got >> 7) != 0, np.signbit(x))


def test_e4m3_clamp_and_specials():
    x = np.array([448.0, 449.0, 1e30, -1e30, np.inf, -np.inf, 0.0, -0.0, np.nan], dtype=np.float32)
    got = O.e4m3_encode(x)
    assert list(got) == [0x7E, 0x7E, 0x7E, 0xFE, 0x7E, 0xFE, 0x00, 0x80, 0x00]


def test_f16_all_patterns_and_rne():
    h = np.arange(65536, dtype=np.uint16)
    f = O.f16_to_f32(h)
    assert np.array_equal(f, h.view(np.float16).astype(np.float32), equal_nan=True)
    finite = ~np.isnan(f)
    assert np.array_equal(O.f32_to_f16(f[finite]), h[finite])
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(200000) * 10.0 ** rng.integers(-9, 6, 200000)).astype(np.float32)
    with np.errstate(over="ignore"):
        assert np.array_equal(O.f32_to_f16(x), x.astype(np.float16).view(np.uint16))


def test_bf16_conversions():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(100000) * 10.0 ** rng.integers(-30, 30, 100000)).astype(np.float32)
    import torch
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16(x), want)
    # f64 -> bf16 with a single rounding equals f32 -> bf16 whenever the f64 value is an f32 value
    assert np.array_equal(O.f64_to_bf16(x.astype(np.float64)), want)
    # a value just above a bf16 midpoint in f64 must round up even though its f32 rounding is the midpoint
    mid = 1.0 + 2.0 ** -8
    assert O.f64_to_bf16(np.array([mid + 2.0 ** -40]))[0] == 0x3F81
    assert O.f64_to_bf16(np.array([mid]))[0] == 0x3F80        # exact tie -> even


def test_int4_round_trip():
    rng = np.random.default_rng(4)
    W = (rng.uniform(-500, 500, (5, 384)) * 1e-4).astype(np.float32)
    p, s = O.quantize_int4_g128(W)
    n = O.unpack_nibbles(p)
    assert n.min() >= 1 and n.max() <= 15
    sf = np.repeat(O.f16_to_f32(s), 128, axis=1)
    assert np.all(np.abs(O.dequant_int4(p, s) - W) <= 0.5 * sf * 1.0001 + 1e-12)


def test_int4_asym_round_trip():
    rng = np.random.default_rng(5)
    W = (rng.standard_normal((7, 512)) * 0.02).astype(np.float32)
    p, s, z = O.quantize_int4_asym(W)
    n = O.unpack_nibbles(p)
    assert n.min() >= 0 and n.max() <= 15
    # bf16 rounding of scale and zero adds at most a few bf16 ulps of the group range on top of half a step
    sf = np.repeat(O.bf16_to_f32(s), 128, axis=1)
    err = np.abs(O.dequant_int4_asym(p, s, z) - W)
    assert np.all(err <= 0.5 * sf + 16 * 2.0 ** -8 * sf * 8)


def test_fp8_round_trip():
    rng = np.random.default_rng(6)
    W = (rng.uniform(-500, 500, (5, 384)) * 1e-4).astype(np.float32)
    q, s = O.quantize_fp8_rowwise(W)
    d = O.dequant_fp8(q, s)
    assert np.all(np.abs(d - W) <= np.abs(W) * 0.0625 + s[:, None] * 2.0 ** -10)
    assert not np.any((q & 0x7F) == 0x7F)


# ---------------------------------------------------------------- against the reference's own compiled code

REF = O.ref_quant_lib()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref not built (no reference checkout on this machine)")


@needs_ref
def test_against_reference_quant_host_bitexact():
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.uniform(-500, 500, 20000), rng.standard_normal(20000) * 1e-4,
                        np.array([0.0, -0.0, 448, 449, np.inf, -np.inf, np.nan])]).astype(np.float32)
    ref = np.array([REF.ref_e4m3_encode(float(v)) for v in x], dtype=np.uint8)
    assert np.array_equal(O.e4m3_encode(x), ref)
    h = np.arange(65536, dtype=np.uint16)
    assert np.array_equal(O.f16_to_f32(h), np.array([REF.ref_f16_to_f32(int(v)) for v in h], np.float32),
                          equal_nan=True)
    y = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    assert np.array_equal(O.f32_to_f16(y), np.array([REF.ref_f32_to_f16(float(v)) for v in y], np.uint16))
    W = (rng.standard_normal((9, 384)) * 0.02).astype(np.float32)
    W[3] = 0.0
    import ctypes
    q1 = np.empty((9, 384), np.uint8); s1 = np.empty(9, np.float32)
    REF.ref_quantize_fp8_rowwise(W.ctypes.data_as(ctypes.c_void_p), 9, 384, q1.ctypes.data_as(ctypes.c_void_p),
                                 s1.ctypes.data_as(ctypes.c_void_p))
    q2, s2 = O.quantize_fp8_rowwise(W)
    assert np.array_equal(q1, q2) and np.array_equal(s1, s2)
    p1 = np.empty((9, 192), np.uint8); c1 = np.empty((9, 3), np.uint16)
    REF.ref_quantize_int4_g128(W.ctypes.data_as(ctypes.c_void_p), 9, 384, p1.ctypes.data_as(ctypes.c_void_p),
                               c1.ctypes.data_as(ctypes.c_void_p))
    p2, c2 = O.quantize_int4_g128(W)
    assert np.array_equal(p1, p2) and np.array_equal(c1, c2)


def test_reference_selftest_binary_passes():
    exe = O.HERE / "_ref" / "quant_host_selftest"
    if not exe.exists():
        pytest.skip("reference self-test not built")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "passed" in r.stdout
