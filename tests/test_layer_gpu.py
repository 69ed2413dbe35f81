"""paia_gemv_layer: one persistent launch for a sequence of GEMVs (a decode layer's projections). Each op is checked
against the CPU oracle on the bytes it actually read (for a chained op, the previous op's output as the layer wrote
it), within the tolerance of the per-format calls; two launches give the same bits (the counters are left zero, so
the second launch waits as the first did); argument errors; replay inside a captured CUDA graph."""

import numpy as np
import pytest
import torch

import oracle as O
from gpu_cases import KINDS, bits, check, make

pytestmark = pytest.mark.gpu

LLAMA = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from paia_gemv import load_lib
    return load_lib()


def _p(t):
    return None if t is None else t.data_ptr()


def op_dict(o, x, y, bias=None):
    return dict(Wq=_p(o.W), scales=_p(o.s), zeros=_p(o.z), x=_p(x), bias=_p(bias), y=_p(y), N=o.N, K=o.K)


def counters(n):
    return torch.zeros(n + 1, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("kind", KINDS)
def test_chained_layer_matches_oracle(L, kind):
    """x of op j is y of op j - 1; the first op has a bias. The x each op read is the previous y as stored, so the
    oracle sees the same bytes."""
    # long rows (several stages per row), then an op with fewer rows than SMs (CTAs without rows)
    shapes = [(1536, 1024), (1024, 1536), (14336, 1024), (128, 14336)]
    ops = [make(kind, N, K, seed=40 + j, with_bias=(j == 0)) for j, (N, K) in enumerate(shapes)]
    ys = [torch.full((o.N,), float("nan"), dtype=torch.bfloat16, device="cuda") for o in ops]
    desc = []
    for j, o in enumerate(ops):
        x = o.x if j == 0 else ys[j - 1]
        desc.append(op_dict(o, x, ys[j], o.bias if j == 0 else None))
    c = counters(len(ops))
    L.layer(kind, desc, c.data_ptr())
    torch.cuda.synchronize()
    assert L.device_error(1) == 0
    assert c.tolist() == [0] * (len(ops) + 1)
    for j, o in enumerate(ops):
        xb = bits(o.x) if j == 0 else bits(ys[j - 1])
        want = o.oracle(with_bias=(j == 0), x_bits=xb)[0]
        check(o, bits(ys[j]), want, f"layer {kind} op {j} {o.N}x{o.K}")


@pytest.mark.parametrize("kind", KINDS)
def test_independent_ops_deterministic(L, kind):
    """Six independent ops (the most one launch takes), ragged and tiny N included; a second launch on the same
    inputs gives the same bits for every op."""
    shapes = [(1000, 2048), (100, 4096), (40, 256), (3000, 128), (2048, 5120), (17, 1024)]
    ops = [make(kind, N, K, seed=60 + j, with_bias=(j % 2 == 1)) for j, (N, K) in enumerate(shapes)]
    c = counters(len(ops))
    runs = []
    for _ in range(2):
        for o in ops:
            o.nan_fill()
        L.layer(kind, [op_dict(o, o.x, o.y, o.bias) for o in ops], c.data_ptr())
        torch.cuda.synchronize()
        assert L.device_error(1) == 0
        runs.append([bits(o.y).copy() for o in ops])
    assert c.tolist() == [0] * (len(ops) + 1)
    for j, o in enumerate(ops):
        assert np.array_equal(runs[0][j], runs[1][j]), f"{kind} op {j}: launches differ"
        check(o, runs[0][j], o.oracle(with_bias=o.bias is not None)[0], f"layer {kind} op {j} {o.N}x{o.K}")


@pytest.mark.parametrize("kind", ["fp8", "int4_asym"])
def test_llama_layer_against_per_op_calls(L, kind):
    """The Llama-3.1-8B projections of one decode layer in one launch: each op within tolerance of the oracle and of
    the per-format call on the same operands."""
    ops = [make(kind, N, K, seed=80 + j) for j, (N, K) in enumerate(LLAMA)]
    c = counters(len(ops))
    L.layer(kind, [op_dict(o, o.x, o.y) for o in ops], c.data_ptr())
    torch.cuda.synchronize()
    assert L.device_error(1) == 0
    from gpu_cases import DEFAULT, variant_id
    v = variant_id(L, kind, DEFAULT[kind])
    for j, o in enumerate(ops):
        got = bits(o.y).copy()
        alone = torch.full((o.N,), float("nan"), dtype=torch.bfloat16, device="cuda")
        o.call(L, v, y=alone)
        torch.cuda.synchronize()
        check(o, got, bits(alone), f"layer vs per-op call {kind} op {j}")
        check(o, got, o.oracle()[0], f"layer {kind} op {j}")


def test_layer_argument_errors(L):
    o = make("fp8", 256, 512, seed=1)
    c = counters(6)
    f = L._lib.paia_gemv_layer
    from paia_gemv.loader import GemvOp
    one = (GemvOp * 7)(*[GemvOp(**op_dict(o, o.x, o.y)) for _ in range(7)])
    assert f(1, 0, 0, one, c.data_ptr(), None) == -2                  # no ops
    assert f(1, 0, 7, one, c.data_ptr(), None) == -2                  # more than six
    assert f(1, 0, 1, one, c.data_ptr() + 2, None) == -2              # misaligned counters
    assert f(1, 0, 1, one, None, None) == -2                          # no counters
    assert f(5, 0, 1, one, c.data_ptr(), None) == -2                  # bad kind
    bad = (GemvOp * 1)(GemvOp(**op_dict(o, o.x, o.x)))               # y overlaps x
    assert f(1, 0, 1, bad, c.data_ptr(), None) == -2
    odd = (GemvOp * 1)(GemvOp(**dict(op_dict(o, o.x, o.y), K=500)))  # K % 16 != 0 for fp8
    assert f(1, 0, 1, odd, c.data_ptr(), None) == -2
    with pytest.raises(ValueError):
        L.layer("fp8", [], c.data_ptr())
    torch.cuda.synchronize()
    assert L.device_error(1) == 0


def test_layer_in_cuda_graph(L):
    """Captured once, replayed on new x contents: outputs follow the inputs, counters stay zero."""
    kind = "fp8"
    shapes = [(2048, 1024), (1024, 2048), (4096, 1024)]
    ops = [make(kind, N, K, seed=90 + j) for j, (N, K) in enumerate(shapes)]
    ys = [torch.empty(o.N, dtype=torch.bfloat16, device="cuda") for o in ops]
    x0 = ops[0].x.clone()
    desc = [op_dict(ops[0], x0, ys[0]), op_dict(ops[1], ys[0], ys[1]), op_dict(ops[2], ops[2].x, ys[2])]
    c = counters(len(ops))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        L.layer(kind, desc, c.data_ptr())                               # warm-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        L.layer(kind, desc, c.data_ptr())
    for seed in (3, 4):
        x0.copy_(make(kind, 8, 1024, seed=seed).x)
        g.replay()
        torch.cuda.synchronize()
        assert L.device_error(1) == 0
        check(ops[0], bits(ys[0]), ops[0].oracle(x_bits=bits(x0))[0], f"graph op 0 seed {seed}")
        check(ops[1], bits(ys[1]), ops[1].oracle(x_bits=bits(ys[0]))[0], f"graph op 1 seed {seed}")
        check(ops[2], bits(ys[2]), ops[2].oracle()[0], f"graph op 2 seed {seed}")
    assert c.tolist() == [0] * (len(ops) + 1)
    del g


def chain_shapes(pairs, head):
    """(N, K) of a chained sequence: each op's K is the previous op's N."""
    out = []
    for n, k in pairs:
        assert not out or out[-1][0] == k
        out.append((n, k))
    out.append(head)
    return out


@pytest.mark.parametrize("kind", KINDS)
def test_plan_whole_token(L, kind):
    """A plan over three small 'layers' (up and down projections, chained) and a head: 7 ops in one launch, checked
    op by op against the oracle on the bytes each op read; launched twice, same bits."""
    pairs = [(3072, 1024), (1024, 3072)] * 3
    shapes = chain_shapes(pairs, (5000, 1024))
    ops = [make(kind, N, K, seed=100 + j) for j, (N, K) in enumerate(shapes)]
    ys = [torch.full((o.N,), float("nan"), dtype=torch.bfloat16, device="cuda") for o in ops]
    desc = [op_dict(o, o.x if j == 0 else ys[j - 1], ys[j]) for j, o in enumerate(ops)]
    plan = L.plan_create(kind, desc)
    try:
        outs = []
        for _ in range(2):
            for y in ys:
                y.fill_(float("nan"))
            L.plan_launch(plan)
            torch.cuda.synchronize()
            assert L.device_error(1) == 0
            outs.append([bits(y).copy() for y in ys])
        for j, o in enumerate(ops):
            assert np.array_equal(outs[0][j], outs[1][j]), f"{kind} op {j}: launches differ"
            xb = bits(o.x) if j == 0 else outs[0][j - 1]
            check(o, outs[0][j], o.oracle(x_bits=xb)[0], f"plan {kind} op {j} {o.N}x{o.K}")
    finally:
        L.plan_destroy(plan)


def test_plan_many_ops_in_graph(L):
    """40 chained ops (more than the 6 a layer launch carries), captured in a CUDA graph and replayed."""
    kind = "int4_asym"
    shapes = [(512, 384) if j % 2 == 0 else (384, 512) for j in range(40)]
    ops = [make(kind, N, K, seed=200 + j) for j, (N, K) in enumerate(shapes)]
    ys = [torch.full((o.N,), float("nan"), dtype=torch.bfloat16, device="cuda") for o in ops]
    x0 = ops[0].x.clone()
    desc = [op_dict(o, x0 if j == 0 else ys[j - 1], ys[j]) for j, o in enumerate(ops)]
    plan = L.plan_create(kind, desc)
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            L.plan_launch(plan)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            L.plan_launch(plan)
        x0.copy_(make(kind, 8, 384, seed=9).x)
        g.replay()
        torch.cuda.synchronize()
        assert L.device_error(1) == 0
        for j in (0, 1, 20, 39):
            xb = bits(x0) if j == 0 else bits(ys[j - 1])
            check(ops[j], bits(ys[j]), ops[j].oracle(x_bits=xb)[0], f"plan op {j}")
        del g
    finally:
        L.plan_destroy(plan)


def test_plan_argument_errors(L):
    from paia_gemv.loader import GemvOp
    import ctypes
    o = make("bf16", 64, 256, seed=2)
    h = ctypes.c_void_p()
    one = (GemvOp * 1)(GemvOp(**op_dict(o, o.x, o.y)))
    f = L._lib.paia_gemv_plan_create
    assert f(0, 0, 0, one, ctypes.byref(h)) == -2 and not h.value
    assert f(0, 0, 4097, one, ctypes.byref(h)) == -2
    assert f(0, 0, 1, one, None) == -2
    assert L._lib.paia_gemv_plan_launch(None, None) == -2
    assert L._lib.paia_gemv_plan_destroy(None) == 0


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("mode", ["layer", "plan"])
def test_fused_silu_mul_between_gate_up_and_down(L, kind, mode):
    """gate_up (2I rows) then down (K = I) reading bf16(SiLU(gate) * up) of gate_up's output, fused into the down
    op's x staging (act = 1): down's output matches the oracle on the activation computed from the stored gate_up
    output."""
    from paia_gemv.loader import GemvOp
    I, H = 1536, 1024
    gu = make(kind, 2 * I, H, seed=300)
    dn = make(kind, H, I, seed=301)
    y_gu = torch.full((2 * I,), float("nan"), dtype=torch.bfloat16, device="cuda")
    y_dn = torch.full((H,), float("nan"), dtype=torch.bfloat16, device="cuda")
    ops = [op_dict(gu, gu.x, y_gu), dict(op_dict(dn, y_gu, y_dn), act=GemvOp.ACT_SILU_MUL)]
    if mode == "layer":
        c = counters(2)
        L.layer(kind, ops, c.data_ptr())
    else:
        plan = L.plan_create(kind, ops)
        L.plan_launch(plan)
    torch.cuda.synchronize()
    if mode == "plan":
        L.plan_destroy(plan)
    assert L.device_error(1) == 0
    check(gu, bits(y_gu), gu.oracle()[0], f"{mode} {kind} gate_up")
    act = O.silu_mul(bits(y_gu))
    check(dn, bits(y_dn), dn.oracle(x_bits=act)[0], f"{mode} {kind} down(silu*mul)")


def test_act_argument_checks(L):
    o = make("fp8", 256, 512, seed=1)
    c = counters(1)
    from paia_gemv.loader import GemvOp
    bad = (GemvOp * 1)(GemvOp(**dict(op_dict(o, o.x, o.y), act=2)))
    assert L._lib.paia_gemv_layer(1, 0, 1, bad, c.data_ptr(), None) == -2
    # with act = 1 x spans 2K values: a y right after the first K values overlaps it
    xx = torch.zeros(2 * 512 + 256, dtype=torch.bfloat16, device="cuda")
    ov = (GemvOp * 1)(GemvOp(**dict(op_dict(o, xx, xx[512:]), act=1)))
    assert L._lib.paia_gemv_layer(1, 0, 1, ov, c.data_ptr(), None) == -2
