"""Parity on realistic decode activations: x with outlier channels (1, 4 or 16 channels at 100x to 10000x the rest,
as LLM activations carry, worst at the down projection's input) and the SiLU(gate) * up activation that feeds the
down projection. The reference's kernels multiply every bf16 x exactly in fp32 (src/paia_gemv/gemv_fp8.cuh:41-52,
gemv_int4.cuh:39-52); the B200 tensor-core paths stage x in parts (FP8: four e4m3 terms in two exponent tiers, INT4:
four int8 digits), so these cases check that no part of x is lost next to an outlier. Every real Llama-3.1-8B and
Qwen2.5-7B decode shape in FP8, INT4 and asymmetric INT4 through the default variant (the path a caller gets), plus
batched x rows; relative L2 <= 1e-3 against the bf16-rounded fp64 oracle on the same bytes (sampled rows for the
large shapes)."""
import numpy as np
import pytest
import torch

import oracle as O
from gpu_cases import DEFAULT, TOL, bits, variant_id
from paia_gemv import quant, synthetic

pytestmark = pytest.mark.gpu

SHAPES = sorted({s for m in synthetic.SHAPES.values() for name, s in m.items()})
OUTLIERS = [(n, mag) for n in (1, 4, 16) for mag in (100.0, 1000.0, 3000.0, 10000.0)]
ROWS = 4096                                                     # oracle rows sampled per shape


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from paia_gemv import load_lib
    return load_lib()


def activation(K, seed, n_out=0, mag=0.0, silu=False):
    """bf16 x [K] on the CPU generator: N(0, 1), or SiLU(g) * u with g, u ~ N(0, 1.28^2) (the gate_up outputs of an
    N(0, 0.02) projection of N(0, 1) x), with n_out channels set to +-mag."""
    g = torch.Generator().manual_seed(seed)
    if silu:
        gate = torch.randn(K, generator=g) * 1.28
        up = torch.randn(K, generator=g) * 1.28
        x = torch.nn.functional.silu(gate) * up
    else:
        x = torch.randn(K, generator=g)
    if n_out:
        idx = torch.randperm(K, generator=g)[:n_out]
        sign = torch.where(torch.rand(n_out, generator=g) < 0.5, -1.0, 1.0)
        x[idx] = sign * mag
    return x.to(torch.bfloat16)


class Weights:
    """Quantised weights of one shape on the device (CUDA generator: the large shapes quantise in seconds), and the
    bytes of the sampled rows on the host for the oracle."""

    def __init__(self, kind, N, K, seed):
        g = torch.Generator(device="cuda").manual_seed(seed)
        W = synthetic.weights_f32(N, K, g, device="cuda")
        self.kind, self.N, self.K = kind, N, K
        self.s = self.z = None
        if kind == "fp8":
            self.W, self.s = quant.quantize_fp8_rowwise(W)
        elif kind == "int4":
            self.W, self.s = quant.quantize_int4_g128(W)
        else:
            self.W, self.s, self.z = quant.quantize_int4_asym(W)
        del W
        rng = np.random.default_rng(seed)
        self.rows = np.arange(N) if N <= ROWS else np.sort(rng.choice(N, ROWS, replace=False))
        idx = torch.as_tensor(self.rows, device="cuda")
        take = lambda t: None if t is None else t.index_select(0, idx).cpu()      # noqa: E731
        self.hW, self.hs, self.hz = take(self.W), take(self.s), take(self.z)

    def oracle(self, x):
        xb = bits(x)
        if self.kind == "fp8":
            return O.gemv("fp8", xb, q=self.hW.numpy(), scale=self.hs.numpy())[0]
        if self.kind == "int4":
            return O.gemv("int4", xb, packed=self.hW.numpy(), scales=bits(self.hs))[0]
        return O.gemv("int4_asym", xb, packed=self.hW.numpy(), scales=bits(self.hs), zeros=bits(self.hz))[0]

    def call(self, L, x):
        y = torch.full((self.N,), float("nan"), dtype=torch.bfloat16, device="cuda")
        v = variant_id(L, self.kind, DEFAULT[self.kind])
        xd = x.cuda()
        if self.kind == "fp8":
            L.fp8(self.W.data_ptr(), self.s.data_ptr(), xd.data_ptr(), y.data_ptr(), self.N, self.K, v)
        elif self.kind == "int4":
            L.int4(self.W.data_ptr(), self.s.data_ptr(), xd.data_ptr(), y.data_ptr(), self.N, self.K, v)
        else:
            L.int4_asym(self.W.data_ptr(), self.s.data_ptr(), self.z.data_ptr(), xd.data_ptr(), y.data_ptr(),
                        self.N, self.K, v)
        torch.cuda.synchronize()
        return bits(y)[self.rows]


def cases(K):
    out = [("N(0,1)", activation(K, 11)), ("silu*up", activation(K, 12, silu=True))]
    for i, (n, mag) in enumerate(OUTLIERS):
        out.append((f"{n}x{mag:g}", activation(K, 100 + i, n, mag)))
    out.append(("silu*up+4x3000", activation(K, 13, 4, 3000.0, silu=True)))
    return out


@pytest.mark.parametrize("kind", ["fp8", "int4", "int4_asym"])
@pytest.mark.parametrize("N,K", SHAPES)
def test_outlier_activations_every_real_shape(L, kind, N, K):
    w = Weights(kind, N, K, seed=N + 3 * K)
    worst = (0.0, "")
    for name, x in cases(K):
        y = w.call(L, x)
        ref = w.oracle(x)
        assert not np.isnan(O.bf16_to_f32(y)).any(), f"{kind} {N}x{K} {name}: unwritten rows"
        err = O.rel_l2(y, ref)
        assert err <= TOL, f"{kind} {N}x{K} x={name}: rel L2 {err:.3e} > {TOL}"
        worst = max(worst, (err, name))
    assert L.device_error(1) == 0
    print(f"{kind} {N}x{K}: worst rel L2 {worst[0]:.2e} ({worst[1]})")


@pytest.mark.parametrize("kind", ["fp8", "int4", "int4_asym"])
@pytest.mark.parametrize("N,K", [(4096, 4096), (3584, 18944)])
def test_outlier_activations_batched_rows(L, kind, N, K):
    """paia_gemv_batched with every x row a different activation: each row against the oracle of its own x."""
    w = Weights(kind, N, K, seed=7 * N + K)
    xs = [x for _, x in cases(K)][:8]
    X = torch.stack(xs).cuda().contiguous()
    M = X.shape[0]
    Y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    p = lambda t: None if t is None else t.data_ptr()          # noqa: E731
    L.batched(kind, p(w.W), p(w.s), p(w.z), X.data_ptr(), None, Y.data_ptr(), M, N, K)
    torch.cuda.synchronize()
    assert L.device_error(1) == 0
    for m in range(M):
        err = O.rel_l2(bits(Y[m])[w.rows], w.oracle(xs[m]))
        assert err <= TOL, f"batched {kind} {N}x{K} row {m}: rel L2 {err:.3e}"
