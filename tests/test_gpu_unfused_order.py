"""Stream order of the unfused INT4 control (src/paia_gemv/gemv_quant.cu:88-97): the dequantisation kernel writes the
bf16 scratch and the BF16 GEMV that follows reads it as its weights. The GEMV must see every byte of the scratch the
dequantisation just wrote, call after call: 500 calls back to back over two alternating operand sets sharing one
scratch (in a CUDA graph for the caller-scratch entry point, eagerly with no host synchronisation for the
library-scratch one), every output equal bit for bit to an isolated call, which itself matches the oracle."""
import numpy as np
import pytest
import torch

import oracle as O
from gpu_cases import bits, check, make

pytestmark = pytest.mark.gpu

N, K, CALLS = 4096, 4096, 500                  # N > 1024: the BF16 stage takes the TMA-fed kernel


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from paia_gemv import load_lib
    return load_lib()


@pytest.fixture(scope="module")
def operands(L):
    ops = [make("int4", N, K, seed=s) for s in (21, 22)]
    scratch = torch.empty(N * K, dtype=torch.bfloat16, device="cuda")
    refs = []
    for o in ops:
        y = torch.full((N,), float("nan"), dtype=torch.bfloat16, device="cuda")
        L.int4_unfused(o.W.data_ptr(), o.s.data_ptr(), o.x.data_ptr(), y.data_ptr(), scratch.data_ptr(), N, K)
        torch.cuda.synchronize()
        refs.append(bits(y))
        # the control rounds the dequantised weights to bf16 before the BF16 GEMV (as gemv_int4.cuh:154-174 does)
        wb = O.dequant_int4_to_bf16(o.W.cpu().numpy(), bits(o.s))
        check(o, refs[-1], O.gemv("bf16", bits(o.x), W=wb)[0], "unfused isolated call")
    return ops, scratch, refs


def test_unfused_graph_replay_alternating_operands(L, operands):
    ops, scratch, refs = operands
    Y = torch.full((CALLS, N), float("nan"), dtype=torch.bfloat16, device="cuda")

    def calls():
        for i in range(CALLS):
            o = ops[i % 2]
            L.int4_unfused(o.W.data_ptr(), o.s.data_ptr(), o.x.data_ptr(), Y[i].data_ptr(), scratch.data_ptr(), N, K)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        calls()                                            # warm-up (and first-call setup) outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        calls()
    for rep in range(2):
        Y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        got = bits(Y)
        for i in range(CALLS):
            assert np.array_equal(got[i], refs[i % 2]), (rep, i)
    del g


def test_unfused_static_back_to_back_alternating_operands(L, operands):
    ops, _, refs = operands
    Y = torch.full((CALLS, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    for i in range(CALLS):
        o = ops[i % 2]
        L.int4_unfused_static(o.W.data_ptr(), o.s.data_ptr(), o.x.data_ptr(), Y[i].data_ptr(), N, K)
    torch.cuda.synchronize()
    got = bits(Y)
    for i in range(CALLS):
        assert np.array_equal(got[i], refs[i % 2]), i
