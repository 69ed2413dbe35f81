"""The oracle's fused-activation step, bf16(SiLU(gate) * up), on known values (no GPU)."""
import math

import numpy as np

import oracle as O


def test_silu_mul_known_values():
    g = np.array([0.0, 1.0, -1.0, 4.0, -100.0, 2.5], dtype=np.float32)
    u = np.array([3.0, 1.0, 2.0, -0.5, 7.0, 1.0], dtype=np.float32)
    bits = O.f32_to_bf16(np.concatenate([g, u]))
    gb, ub = O.bf16_to_f32(bits[:6]).astype(np.float64), O.bf16_to_f32(bits[6:]).astype(np.float64)
    got = O.bf16_to_f32(O.silu_mul(bits)).astype(np.float64)
    want = np.array([gv / (1 + math.exp(-gv)) * uv for gv, uv in zip(gb, ub)])
    assert got[0] == 0.0 and got[4] == 0.0                     # SiLU(0) = 0; SiLU(-100) * 7 rounds to -0 in bf16
    assert np.allclose(got, want, rtol=2 ** -8, atol=1e-38)     # one bf16 rounding (below bf16 range: 0)
    assert abs(got[1] - 0.7310585786) < 2 ** -8


def test_silu_mul_length_and_rounding():
    rng = np.random.default_rng(3)
    gu = O.f32_to_bf16(rng.standard_normal(2 * 1024).astype(np.float32))
    y = O.silu_mul(gu)
    assert y.shape == (1024,) and y.dtype == np.uint16
    # exactly the bf16 rounding of the fp64 value
    g = O.bf16_to_f32(gu[:1024]).astype(np.float64)
    u = O.bf16_to_f32(gu[1024:]).astype(np.float64)
    assert np.array_equal(y, O.f64_to_bf16(g / (1 + np.exp(-g)) * u))
