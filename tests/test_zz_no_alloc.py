"""paia_gemv_int4_unfused_static is the unfused INT4 control for callers that cannot hand the library a scratch
buffer: a serving engine whose memory pool already owns the whole HBM budget, a plain C host with no device
allocator of its own, or a latency-critical loop where cudaMalloc / cudaFree would synchronise the device. It
dequantises into the library's own file-scope device array instead, so a call allocates nothing.

Checked through the C ABI against paia_gemv_int4_unfused with a caller-owned scratch: the same output bytes on two
calls in a row (the second call reuses the array the first one filled), and a clear -2 (a RuntimeError from the
Python binding) for N x K beyond the array's 16 Mi elements. The file name sorts last, so a run that stops at the
first failure has run every other test first; the test passes alone in a fresh process as well as after the rest."""
import numpy as np
import pytest
import torch

from gpu_cases import bits, make

pytestmark = pytest.mark.gpu

STATIC_ELEMS = 16 << 20


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from paia_gemv import load_lib
    return load_lib()


def unfused_ref(L, ops):
    scratch = torch.empty(ops.N * ops.K, dtype=torch.bfloat16, device="cuda")
    y = torch.full((ops.N,), float("nan"), dtype=torch.bfloat16, device="cuda")
    L.int4_unfused(ops.W.data_ptr(), ops.s.data_ptr(), ops.x.data_ptr(), y.data_ptr(), scratch.data_ptr(),
                   ops.N, ops.K)
    torch.cuda.synchronize()
    return bits(y)


@pytest.mark.parametrize("N,K", [(33, 1152), (512, 4096), (4096, 4096)])
def test_static_scratch_matches_caller_scratch_twice(L, N, K):
    """Two calls in a row on different operands: each equals the caller-scratch entry point bit for bit (the second
    call also proves the first call's scratch contents do not leak into it). 4096 x 4096 fills the scratch exactly."""
    for seed in (N + K, N + K + 1):
        ops = make("int4", N, K, seed=seed)
        want = unfused_ref(L, ops)
        y = torch.full((N,), float("nan"), dtype=torch.bfloat16, device="cuda")
        L.int4_unfused_static(ops.W.data_ptr(), ops.s.data_ptr(), ops.x.data_ptr(), y.data_ptr(), N, K)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y), want), (N, K, seed)


def test_static_scratch_rejects_oversize(L):
    """N * K above the 16 Mi-element scratch: -2 from the C ABI before any launch, a clear error from Python."""
    N, K = 4097, 4096
    assert N * K > STATIC_ELEMS
    ops = make("int4", 8, 128, seed=3)                  # any valid pointers; nothing is launched
    rc = L._lib.paia_gemv_int4_unfused_static(ops.W.data_ptr(), ops.s.data_ptr(), ops.x.data_ptr(),
                                              ops.y.data_ptr(), N, K, None)
    assert rc == -2
    with pytest.raises(RuntimeError, match="exceeds the static scratch"):
        L.int4_unfused_static(ops.W.data_ptr(), ops.s.data_ptr(), ops.x.data_ptr(), ops.y.data_ptr(), N, K)
