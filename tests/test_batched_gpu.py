"""paia_gemv_batched: Y[M, N] = X[M, K] . W^T (+ bias) with the x rows in the tensor-core MMA columns. Every output
row is checked against the CPU oracle of its own x row (the per-format tolerance), for M from 1 to 17 (one, several
and partial groups of 8 rows), ragged N, long K (groups narrowed by shared memory, and a single-row fallback), and a
bias on every row; plus argument errors."""
import numpy as np
import pytest
import torch

from gpu_cases import KINDS, bits, check, make

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from paia_gemv import load_lib
    return load_lib()


def _p(t):
    return None if t is None else t.data_ptr()


def run_batched(L, o, X, bias=None):
    M = X.shape[0]
    Y = torch.full((M, o.N), float("nan"), dtype=torch.bfloat16, device="cuda")
    L.batched(o.kind, _p(o.W), _p(o.s), _p(o.z), X.data_ptr(), _p(bias), Y.data_ptr(), M, o.N, o.K)
    torch.cuda.synchronize()
    assert L.device_error(1) == 0
    return Y


def x_rows(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g).to(torch.bfloat16).cuda().contiguous()


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("M", [1, 2, 5, 8, 9, 16, 17])
def test_batched_rows_match_oracle(L, kind, M):
    o = make(kind, 1000, 2048, seed=400 + M)
    X = x_rows(M, 2048, seed=M)
    Y = run_batched(L, o, X)
    for m in range(M):
        check(o, bits(Y[m]), o.oracle(x_bits=bits(X[m]))[0], f"batched {kind} M={M} row {m}")


@pytest.mark.parametrize("kind", KINDS)
def test_batched_long_k_and_bias(L, kind):
    """K = 14336: groups of fewer than 8 rows; bias added to every row; ragged N."""
    o = make(kind, 300, 14336, seed=7, with_bias=True)
    X = x_rows(11, 14336, seed=3)
    Y = run_batched(L, o, X, bias=o.bias)
    for m in range(11):
        check(o, bits(Y[m]), o.oracle(with_bias=True, x_bits=bits(X[m]))[0], f"batched long K {kind} row {m}")


@pytest.mark.parametrize("kind", ["bf16", "fp8"])
def test_batched_ragged_k(L, kind):
    """K not a multiple of a 64-byte step (BF16 K % 32 = 8, FP8 K % 64 = 16): the ragged last step reads zeros."""
    K = 4104 if kind == "bf16" else 4112
    o = make(kind, 777, K, seed=9)
    X = x_rows(6, K, seed=4)
    Y = run_batched(L, o, X)
    for m in range(6):
        check(o, bits(Y[m]), o.oracle(x_bits=bits(X[m]))[0], f"batched ragged K {kind} row {m}")


def test_batched_special_values(L):
    """x rows of very different magnitudes and an all-zero row: each row's own x scale keeps it exact."""
    o = make("fp8", 512, 4096, seed=11)
    X = x_rows(4, 4096, seed=5)
    X[1] *= 1e-20
    X[2] *= 1e20
    X[3] = 0
    Y = run_batched(L, o, X)
    for m in range(3):
        check(o, bits(Y[m]), o.oracle(x_bits=bits(X[m]))[0], f"batched range row {m}")
    assert np.all(bits(Y[3]) & 0x7FFF == 0)


def test_batched_argument_errors(L):
    o = make("int4", 64, 256, seed=1)
    X = x_rows(2, 256, seed=1)
    Y = torch.empty(2, 64, dtype=torch.bfloat16, device="cuda")
    f = L._lib.paia_gemv_batched
    assert f(2, _p(o.W), _p(o.s), None, X.data_ptr(), None, Y.data_ptr(), 0, 64, 256, None) == -2      # M = 0
    assert f(7, _p(o.W), _p(o.s), None, X.data_ptr(), None, Y.data_ptr(), 2, 64, 256, None) == -2      # bad kind
    assert f(2, _p(o.W), _p(o.s), None, X.data_ptr(), None, Y.data_ptr(), 2, 64, 200, None) == -2      # K % 128
    with pytest.raises(RuntimeError):
        L.batched("int4", _p(o.W), _p(o.s), None, X.data_ptr() + 2, None, Y.data_ptr(), 2, 64, 256)   # x unaligned
