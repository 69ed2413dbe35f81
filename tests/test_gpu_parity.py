"""GPU parity of the B200 kernels against the CPU oracle (relative L2 <= 1e-3 against the bf16-rounded fp64
dequantise-then-matmul result), through the C ABI, on the reference's test shapes (src/tests/test_gemv_bf16.py:16-19,
gemv_bf16_check.cu:55-63): awkward shapes for every variant, every real Llama-3.1-8B / Qwen2.5-7B decode shape for
the default variants, the fused and lm_head shapes with sampled rows plus exact size-independent properties. Every
output buffer is prefilled with NaN so an unwritten row fails."""
import numpy as np
import pytest
import torch

import oracle as O
from test_kernel_mapping import share_cap, tma_prep
from gpu_cases import DEFAULT, KINDS, Operands, bits, check, lib, make, variant_id
from paia_gemv import quant, synthetic

pytestmark = pytest.mark.gpu

AWKWARD = {"bf16": [(1, 8), (1, 256), (3, 264), (7, 520), (33, 1032), (129, 4104), (1000, 3584), (513, 14336)],
           "fp8": [(1, 16), (3, 272), (7, 528), (33, 1040), (129, 4112), (1000, 3584), (513, 14336)],
           "int4": [(1, 128), (3, 256), (7, 640), (33, 1152), (129, 4224), (1000, 3584), (513, 14336)]}
AWKWARD["int4_asym"] = AWKWARD["int4"]
REAL = sorted({s for m in synthetic.SHAPES.values() for name, s in m.items() if name != "lm_head"})
BIG = [(128256, 4096), (152064, 3584), (28672, 4096), (37888, 3584)]


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return lib()


def table(L, kind):
    return {"bf16": L.variants, "fp8": L.variants_fp8, "int4": L.variants_int4, "int4_asym": L.variants_int4_asym}[kind]


@pytest.mark.parametrize("kind", KINDS)
def test_every_variant_awkward_shapes(L, kind):
    for (N, K) in AWKWARD[kind]:
        ops = make(kind, N, K, seed=N * 7 + K, with_bias=True)
        ref, _ = ops.oracle()
        refb, _ = ops.oracle(with_bias=True)
        for v in table(L, kind):
            ops.nan_fill()
            ops.call(L, v["id"], bias=None if v["id"] % 2 else ops.bias)
            torch.cuda.synchronize()
            want = ref if v["id"] % 2 else refb
            check(ops, bits(ops.y), want, f"{kind} {N}x{K} variant {v}")


@pytest.mark.parametrize("kind", KINDS)
def test_real_shapes_default_variant(L, kind):
    v = variant_id(L, kind, DEFAULT[kind])
    for (N, K) in REAL:
        if kind != "bf16" and K % (16 if kind == "fp8" else 128):
            continue
        ops = make(kind, N, K, seed=N + K, with_bias=True)
        ops.nan_fill()
        ops.call(L, v)
        torch.cuda.synchronize()
        ref, refd = ops.oracle()
        check(ops, bits(ops.y), ref, f"{kind} {N}x{K}")
        assert O.max_rel(bits(ops.y), refd) < 2e-2      # the reference harness's own gate
        ops.nan_fill()
        ops.call(L, v, bias=ops.bias)
        torch.cuda.synchronize()
        check(ops, bits(ops.y), ops.oracle(with_bias=True)[0], f"{kind} {N}x{K} +bias")


@pytest.mark.parametrize("kind", KINDS)
def test_big_shapes_sampled_rows_and_exact_properties(L, kind):
    """lm_head / fused gate_up at full size: 4096 sampled rows (first, last, random) against the oracle, plus two
    properties that must hold bit for bit at any size: y(2^k x) == 2^k y(x) (power-of-two scaling is exact through
    bf16 products, fp32 sums and the final rounding), and permuting rows of W permutes y."""
    v = variant_id(L, kind, DEFAULT[kind])
    g = torch.Generator(device="cuda").manual_seed(0)
    for (N, K) in BIG:
        W = synthetic.weights_f32(N, K, g, device="cuda")
        x = synthetic.activation_bf16(K, g, device="cuda")
        ops = Operands(kind, W, x)
        del W
        ops.call(L, v)
        torch.cuda.synchronize()
        y0 = bits(ops.y)
        rows = np.unique(np.concatenate([np.arange(64), np.arange(N - 64, N),
                                         np.random.default_rng(N).integers(0, N, 4096)]))
        ref, _ = ops.oracle(rows=rows)
        check(ops, y0[rows], ref, f"{kind} {N}x{K} sampled")
        x4 = (ops.x.float() * 4).to(torch.bfloat16)
        y4 = torch.empty_like(ops.y)
        ops.call(L, v, y=y4, x=x4)
        torch.cuda.synchronize()
        assert torch.equal(y4, (ops.y.float() * 4).to(torch.bfloat16)), f"{kind} {N}x{K}: scaling property"
        if kind == "bf16":
            perm = torch.randperm(N, device="cuda", generator=g)
            yp = torch.empty_like(ops.y)
            Wp = ops.W[perm].contiguous()
            L.bf16(Wp.data_ptr(), ops.x.data_ptr(), yp.data_ptr(), N, K, v)
            torch.cuda.synchronize()
            assert torch.equal(yp, ops.y[perm]), "row permutation property"
        del ops
        torch.cuda.empty_cache()


def test_golden_vectors_on_gpu(L, golden):
    """The reference's own quantised bytes (tests/golden): the kernels agree with the reference harness's fp32
    result and with the reference kernels' emulated result, within the parity tolerance."""
    for name in [str(c) for c in golden["cases"]]:
        x = torch.from_numpy(golden[f"{name}/x"].view(np.int16)).view(torch.bfloat16).cuda()
        if name.startswith("bf16") or name.startswith("special"):
            if f"{name}/W" in golden.files:
                Wb = torch.from_numpy(golden[f"{name}/W"].view(np.int16)).view(torch.bfloat16).cuda()
            else:
                N, K = map(int, name.split("_")[1].split("x"))
                Wb = synthetic.operands(N, K, seed=int(name.split("_s")[-1]))[0].to(torch.bfloat16).cuda()
            kind, args = "bf16", (Wb,)
        elif name.startswith("fp8"):
            kind, args = "fp8", (torch.from_numpy(golden[f"{name}/q"]).cuda(), torch.from_numpy(golden[f"{name}/scale"]).cuda())
        elif name.startswith("int4a"):
            kind = "int4_asym"
            args = (torch.from_numpy(golden[f"{name}/packed"]).cuda(),
                    torch.from_numpy(golden[f"{name}/scales"].view(np.int16)).view(torch.bfloat16).cuda(),
                    torch.from_numpy(golden[f"{name}/zeros"].view(np.int16)).view(torch.bfloat16).cuda())
        else:
            kind = "int4"
            args = (torch.from_numpy(golden[f"{name}/packed"]).cuda(),
                    torch.from_numpy(golden[f"{name}/scales"].view(np.int16)).view(torch.float16).cuda())
        N = args[0].shape[0]
        K = x.shape[0]
        y = torch.full((N,), float("nan"), device="cuda", dtype=torch.bfloat16)
        vid = variant_id(L, kind, DEFAULT[kind])
        if kind == "bf16":
            L.bf16(args[0].data_ptr(), x.data_ptr(), y.data_ptr(), N, K, vid)
        elif kind == "fp8":
            L.fp8(args[0].data_ptr(), args[1].data_ptr(), x.data_ptr(), y.data_ptr(), N, K, vid)
        elif kind == "int4":
            L.int4(args[0].data_ptr(), args[1].data_ptr(), x.data_ptr(), y.data_ptr(), N, K, vid)
        else:
            L.int4_asym(args[0].data_ptr(), args[1].data_ptr(), args[2].data_ptr(), x.data_ptr(), y.data_ptr(), N, K, vid)
        torch.cuda.synchronize()
        yb = bits(y)
        ref = golden[f"{name}/y_ref_fp32"]
        if np.all(ref == 0):
            assert np.all(O.bf16_to_f32(yb) == 0), name
            continue
        check(None, yb, O.f32_to_bf16(ref), f"golden {name} vs reference fp32")
        if f"{name}/y_refkernel_fp32" in golden.files:
            check(None, yb, O.f32_to_bf16(golden[f"{name}/y_refkernel_fp32"]), f"golden {name} vs reference kernel")


def test_fp8_every_code_exact(L):
    """Row c holds e4m3 code c at column c % 16 and zeros elsewhere, x = 1, scale = 1: y must be the code's value
    exactly (all 254 finite codes, both halves of every 16-bit word, every byte of the chunk)."""
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    N, K = len(codes), 64
    q = np.zeros((N, K), np.uint8)
    q[np.arange(N), np.arange(N) % K] = codes
    s = np.ones(N, np.float32)
    x = torch.ones(K, dtype=torch.bfloat16, device="cuda")
    y = torch.full((N,), float("nan"), device="cuda", dtype=torch.bfloat16)
    qd, sd = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    for v in L.variants_fp8:
        y.fill_(float("nan"))
        L.fp8(qd.data_ptr(), sd.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, v["id"])
        torch.cuda.synchronize()
        # compared as values: code 0x80 (-0.0) sums to +0.0, which is the same number
        want = O.bf16_to_f32(O.f32_to_bf16(O.e4m3_decode(codes)))
        assert np.array_equal(O.bf16_to_f32(bits(y)), want), v


@pytest.mark.parametrize("kind", ["int4", "int4_asym"])
def test_int4_every_nibble_position_exact(L, kind):
    """Each row has one nonzero position (every k mod 32, every nibble value 0..15) with scale 1 (and zero 0):
    y = (n - 8) * x[k] exactly, which pins the nibble order of the packed format on the device."""
    K = 256
    rows = [(k, n) for k in range(32) for n in range(16)]
    N = len(rows)
    q = np.full((N, K), 8, np.int64)
    for i, (k, n) in enumerate(rows):
        q[i, k + 32 * (i % 8)] = n
    packed = quant.pack_nibbles(torch.from_numpy(q)).cuda()
    x = torch.arange(1, K + 1, dtype=torch.float32).to(torch.bfloat16).cuda()
    y = torch.full((N,), float("nan"), device="cuda", dtype=torch.bfloat16)
    G = K // 128
    for v in (L.variants_int4 if kind == "int4" else L.variants_int4_asym):
        y.fill_(float("nan"))
        if kind == "int4":
            s = torch.ones(N, G, dtype=torch.float16, device="cuda")
            L.int4(packed.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, v["id"])
        else:
            s = torch.ones(N, G, dtype=torch.bfloat16, device="cuda")
            z = torch.zeros(N, G, dtype=torch.bfloat16, device="cuda")
            L.int4_asym(packed.data_ptr(), s.data_ptr(), z.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, v["id"])
        torch.cuda.synchronize()
        want = np.array([(n - 8) * float(x[k + 32 * (i % 8)]) for i, (k, n) in enumerate(rows)], np.float32)
        assert np.array_equal(bits(y), O.f32_to_bf16(want)), v


def test_special_values(L, golden):
    """Zero weights and large-magnitude weights and activations (src/tests/test_gemv_bf16.py:26-29)."""
    for name in ("special_zeros", "special_large"):
        W = torch.from_numpy(golden[f"{name}/W"].view(np.int16)).view(torch.bfloat16).cuda()
        x = torch.from_numpy(golden[f"{name}/x"].view(np.int16)).view(torch.bfloat16).cuda()
        N, K = W.shape
        for v in L.variants:
            y = torch.full((N,), float("nan"), device="cuda", dtype=torch.bfloat16)
            L.bf16(W.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, v["id"])
            torch.cuda.synchronize()
            ref, _ = O.gemv("bf16", golden[f"{name}/x"], W=golden[f"{name}/W"])
            if name == "special_zeros":
                assert np.all(O.bf16_to_f32(bits(y)) == 0)
            else:
                check(None, bits(y), ref, f"{name} {v}")


def test_controls_naive_and_unfused(L):
    for (N, K) in [(7, 640), (513, 3584), (4096, 4096)]:
        ops = make("int4", N, K, seed=3)
        ref, _ = ops.oracle()
        ops.nan_fill()
        L.int4_naive(ops.W.data_ptr(), ops.s.data_ptr(), ops.x.data_ptr(), ops.y.data_ptr(), N, K)
        torch.cuda.synchronize()
        check(ops, bits(ops.y), ref, f"naive {N}x{K}")
        scratch = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
        ops.nan_fill()
        L.int4_unfused(ops.W.data_ptr(), ops.s.data_ptr(), ops.x.data_ptr(), ops.y.data_ptr(), scratch.data_ptr(), N, K)
        torch.cuda.synchronize()
        deq = O.dequant_int4_to_bf16(ops.W.cpu().numpy(), bits(ops.s))
        assert np.array_equal(bits(scratch), deq), "unfused stage 1 must equal the bf16-rounded dequantisation"
        check(ops, bits(ops.y), O.gemv("bf16", bits(ops.x), W=deq)[0], f"unfused {N}x{K}")


def test_contract_raises(L):
    W = torch.zeros(4, 12, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        L.bf16(W.data_ptr(), W.data_ptr(), W.data_ptr(), 4, 12, 0)
    big = torch.zeros(131072, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):       # x does not fit in shared memory: rejected, not mis-computed
        L.bf16(big.data_ptr(), big.data_ptr(), big.data_ptr(), 1, 131072, 0)


@pytest.mark.parametrize("kind", KINDS)
def test_long_rows_near_smem_limit(L, kind):
    ops = make(kind, 5, 65536, seed=9)
    ops.call(L, variant_id(L, kind, DEFAULT[kind]))
    torch.cuda.synchronize()
    check(ops, bits(ops.y), ops.oracle()[0], f"{kind} 5x65536")


@pytest.mark.parametrize("kind", KINDS)
def test_launch_ex_explicit_configs(L, kind):
    ops = make(kind, 1000, 4096, seed=11, with_bias=True)
    ref = ops.oracle(with_bias=True)[0]
    maths = (0, 1) if kind != "fp8" else (0,)
    for R, U, Wn, math, pdl, ks, cps in [(1, 1, 4, m, 0, 1, 1) for m in maths] + \
                                         [(2, 2, 8, m, 1, 8, 2) for m in maths] + \
                                         [(4, 1, 8, m, 1, 2, 3) for m in maths] + [(2, 1, 8, maths[-1], 1, 4, 1)] + \
                                         [(1, 2, 8, 2, 1, 0, 0), (1, 4, 16, 2, 0, 0, 2)]:
        ops.nan_fill()
        rc = ops.call_ex(L, R, U, Wn, math, pdl, ks, cps, with_bias=True)
        assert rc == 0, (R, U, Wn, math, pdl, ks, cps, rc)
        torch.cuda.synchronize()
        check(ops, bits(ops.y), ref, f"{kind} ex {(R, U, Wn, math, pdl, ks, cps)}")


@pytest.mark.parametrize("kind", KINDS)
def test_dependent_chain_in_cuda_graph(L, kind):
    """A chain of GEMVs where each one's x is the previous one's y, launched with PDL (H = 1) and captured in a CUDA
    graph: the kernels read their weights before griddepcontrol.wait but x only after it, so the graph must produce
    exactly the eagerly-synchronised chain's result, and that result must match the oracle chain."""
    K = 2048
    vid = variant_id(L, kind, DEFAULT[kind])
    layers = [make(kind, K, K, seed=100 + i) for i in range(6)]
    x0 = synthetic.activation_bf16(K, synthetic.generator(7), device="cpu").cuda()
    ys = [torch.empty(K, dtype=torch.bfloat16, device="cuda") for _ in layers]

    def chain(stream=None):
        x = x0
        for ops, y in zip(layers, ys):
            ops.call(L, vid, y=y, x=x, stream=stream)
            x = y

    chain()
    torch.cuda.synchronize()
    eager = [bits(y) for y in ys]
    # oracle chain on the device's own intermediate values (each step checked on its own input)
    xb = bits(x0)
    for ops, yb in zip(layers, eager):
        check(ops, yb, ops.oracle(x_bits=xb)[0], f"{kind} chain step")
        xb = yb
    for y in ys:
        y.fill_(float("nan"))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    for y in ys:
        y.fill_(float("nan"))
    with torch.cuda.graph(g):
        chain()
    for _ in range(3):
        for y in ys:
            y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for y, e in zip(ys, eager):
            assert np.array_equal(bits(y), e), f"{kind}: graph/PDL chain differs from the eager chain"
    del g


MMA_CFGS = [(1, 4), (2, 8), (4, 8), (2, 16), (4, 16)]      # (U, W) of the tensor-core kernel (math 2)


MMA_MATHS = [("bf16", 2), ("fp8", 2), ("fp8", 3), ("fp8", 4), ("int4", 2), ("int4_asym", 2)]


@pytest.mark.parametrize("kind,math", MMA_MATHS)
def test_mma_kernel_awkward_and_real_shapes(L, kind, math):
    """The tensor-core kernel (gemv_mma.cuh) through paia_gemv_launch_ex: awkward shapes (partial 64-byte steps,
    partial 16-row tiles, fewer rows than CTAs), real decode shapes, with and without bias, PDL on and off; for FP8
    every weight decoder (math 2: cvt, 3: ALU bit decode, 4: split)."""
    shapes = AWKWARD[kind] + [(4096, 4096), (6144, 4096), (3584, 18944), (512, 3584)]
    for (N, K) in shapes:
        ops = make(kind, N, K, seed=N * 3 + K, with_bias=True)
        ref, refb = ops.oracle()[0], ops.oracle(with_bias=True)[0]
        for i, (U, Wn) in enumerate(MMA_CFGS):
            for cps in (0, 1):
                ops.nan_fill()
                rc = ops.call_ex(L, 1, U, Wn, math, (i + cps) % 2, 0, cps, with_bias=bool(cps))
                assert rc == 0, (kind, N, K, U, Wn, cps, rc)
                torch.cuda.synchronize()
                check(ops, bits(ops.y), refb if cps else ref, f"mma {kind} {N}x{K} U{U} W{Wn} cps{cps}")


@pytest.mark.parametrize("scale", [1e-30, 1e-6, 1.0, 3e3, 1e30])
def test_fp8_mma_activation_ranges(L, scale):
    """The FP8 tensor-core path stages x as f16 scaled by a per-launch power of two: tiny, huge and outlier-dominated
    activations must still match the oracle."""
    N, K = 300, 4096
    ops = make("fp8", N, K, seed=5)
    xf = ops.x.float() * scale
    if scale == 1e30:
        xf[17] = 3e38                                      # one outlier near the top of the bf16 range
    ops.x = xf.to(torch.bfloat16)
    ref = ops.oracle()[0]
    for U, Wn in MMA_CFGS:
        for math in (2, 3, 4):
            ops.nan_fill()
            assert ops.call_ex(L, 1, U, Wn, math, 1, 0, 0) == 0
            torch.cuda.synchronize()
            check(ops, bits(ops.y), ref, f"fp8 mma{math} x*{scale}")


@pytest.mark.parametrize("math", [2, 3, 4])
def test_fp8_mma_every_code_exact(L, math):
    """Every finite e4m3 code (subnormal codes included, which the ALU decode turns into f16 subnormals) through the
    tensor-core FP8 kernel: row c holds code c once, x = 1, scale = 1, so y is the code's value exactly."""
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    N, K = len(codes), 64
    q = np.zeros((N, K), np.uint8)
    q[np.arange(N), np.arange(N) % K] = codes
    ops = make("fp8", N, K)
    ops.W = torch.from_numpy(q).cuda()
    ops.s = torch.ones(N, device="cuda")
    ops.x = torch.ones(K, dtype=torch.bfloat16, device="cuda")
    want = O.bf16_to_f32(O.f32_to_bf16(O.e4m3_decode(codes)))
    for U, Wn in MMA_CFGS:
        ops.nan_fill()
        assert ops.call_ex(L, 1, U, Wn, math, 1, 0, 0) == 0
        torch.cuda.synchronize()
        assert np.array_equal(O.bf16_to_f32(bits(ops.y)), want), (math, U, Wn)


# (ring stages (0 = as many as fit), U, NC consumer warps, shared-memory share) of the TMA-fed kernel, math 5-7
TMA_CFGS = [(2, 2, 4, 1), (3, 4, 8, 1), (0, 2, 8, 2), (0, 4, 4, 1), (16, 2, 8, 1), (0, 2, 16, 1)]


def tma_fits(kind, math, NC, N, K, ring, share):
    """Whether the TMA kernel can stage this shape (the CPU mirror of its shared-memory plan); else the C ABI
    returns -2."""
    dec = 2 if (kind.startswith("int4") and math == 7) else (3 if (kind == "fp8" and math == 8) else 0)
    return tma_prep(kind, NC, K, ring, share_cap(share), dec) is not None


TMA_MATHS = [("bf16", 5), ("fp8", 5), ("fp8", 6), ("fp8", 7), ("fp8", 8), ("int4", 5), ("int4", 6), ("int4", 7),
             ("int4_asym", 5), ("int4_asym", 6), ("int4_asym", 7)]


@pytest.mark.parametrize("kind,math", TMA_MATHS)
def test_tma_kernel_awkward_and_real_shapes(L, kind, math):
    """The TMA-fed tensor-core kernel (gemv_tma.cuh) through paia_gemv_launch_ex: awkward shapes (ragged last chunk of
    a row, partial 16-row tiles, fewer rows than CTAs, rows split into several stages), real decode shapes, with and
    without bias, PDL on and off, one and two CTAs per SM; no bounded wait may give up."""
    shapes = AWKWARD[kind] + [(4096, 4096), (6144, 4096), (3584, 18944), (512, 3584), (37, 28672)]
    L.device_error(1)
    for (N, K) in shapes:
        ops = make(kind, N, K, seed=N * 5 + K, with_bias=True)
        ref, refb = ops.oracle()[0], ops.oracle(with_bias=True)[0]
        for i, (ring, U, NC, share) in enumerate(TMA_CFGS):
            if ring == 16 and K > 4096:
                continue                                       # 16 stages of long rows do not fit
            for cps in (0, 1):
                ops.nan_fill()
                rc = ops.call_ex(L, ring, U, NC, math, (i + cps) % 2, share, cps, with_bias=bool(cps))
                if not tma_fits(kind, math, NC, N, K, ring, share):
                    assert rc == -2, (kind, N, K, ring, share, rc)
                    continue
                assert rc == 0, (kind, N, K, ring, U, NC, share, cps, rc)
                torch.cuda.synchronize()
                check(ops, bits(ops.y), refb if cps else ref,
                      f"tma {kind} {N}x{K} ring{ring} U{U} NC{NC} share{share} cps{cps}")
    assert L.device_error(1) == 0


@pytest.mark.parametrize("kind", ["bf16", "fp8", "int4", "int4_asym"])
def test_tma_kernel_long_rows(L, kind):
    """Rows longer than a stage (K up to the C ABI's maximum of 98304): each row is streamed as several chunks, and the
    ring shrinks to fit next to x in shared memory."""
    for K in (65536, 98304):
        N = 40
        ops = make(kind, N, K, seed=K + 1, with_bias=True)
        refb = ops.oracle(with_bias=True)[0]
        for ring, U, NC, share in ((2, 2, 4, 1), (0, 4, 8, 1), (0, 2, 8, 2)):
            ops.nan_fill()
            rc = ops.call_ex(L, ring, U, NC, 5, 1, share, 0, with_bias=True)
            if share == 2 and 2 * K > 115200:
                assert rc == -2                                # x alone (2 K bytes) exceeds half an SM
                continue
            assert rc == 0, (kind, K, ring, share, rc)
            torch.cuda.synchronize()
            check(ops, bits(ops.y), refb, f"tma {kind} K={K} ring{ring} share{share}")
    assert L.device_error(1) == 0


@pytest.mark.parametrize("scale", [1e-30, 1.0, 1e30])
def test_fp8_tma_activation_ranges(L, scale):
    N, K = 300, 4096
    ops = make("fp8", N, K, seed=6)
    xf = ops.x.float() * scale
    if scale == 1e30:
        xf[17] = 3e38
    ops.x = xf.to(torch.bfloat16)
    ref = ops.oracle()[0]
    for ring, U, NC, share in TMA_CFGS:
        for math in (5, 6, 7, 8):
            ops.nan_fill()
            assert ops.call_ex(L, ring, U, NC, math, 1, share, 0) == 0
            torch.cuda.synchronize()
            check(ops, bits(ops.y), ref, f"fp8 tma{math} x*{scale}")


@pytest.mark.parametrize("math", [5, 6, 7, 8])
def test_fp8_tma_every_code_exact(L, math):
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    N, K = len(codes), 64
    q = np.zeros((N, K), np.uint8)
    q[np.arange(N), np.arange(N) % K] = codes
    ops = make("fp8", N, K)
    ops.W = torch.from_numpy(q).cuda()
    ops.s = torch.ones(N, device="cuda")
    ops.x = torch.ones(K, dtype=torch.bfloat16, device="cuda")
    want = O.bf16_to_f32(O.f32_to_bf16(O.e4m3_decode(codes)))
    for ring, U, NC, share in TMA_CFGS:
        ops.nan_fill()
        assert ops.call_ex(L, ring, U, NC, math, 1, share, 0) == 0
        torch.cuda.synchronize()
        assert np.array_equal(O.bf16_to_f32(bits(ops.y)), want), (math, ring, U, NC, share)


@pytest.mark.parametrize("kind,math", [("bf16", 5), ("fp8", 8), ("int4", 7), ("int4_asym", 7)])
def test_tma_tensor_copies_equal_row_copies(L, kind, math):
    """Full tiles as one tiled tensor copy per stage (paia_gemv_launch_ex, ks bit 16) give the same bits as the
    per-row bulk copies: whole rows, chunked rows and a partial last tile per CTA."""
    for (N, K) in ((4096, 4096), (300, 14336), (1000, 3584), (37, 18944)):
        ops = make(kind, N, K, seed=N + 11 * K, with_bias=True)
        outs = []
        for ks in (0, 1 << 16):
            ops.nan_fill()
            assert ops.call_ex(L, 0, 2, 8, math, 1, ks, 0, with_bias=True) == 0
            torch.cuda.synchronize()
            outs.append(bits(ops.y).copy())
        assert np.array_equal(outs[0], outs[1]), (kind, N, K)
        check(ops, outs[1], ops.oracle(with_bias=True)[0], f"tensor copies {kind} {N}x{K}")
    assert L.device_error(1) == 0


@pytest.mark.parametrize("kind", ["bf16", "fp8", "int4", "int4_asym"])
def test_rope_epilogue_matches_oracle(L, kind):
    """paia_gemv_rope: a Qwen-like fused QKV (28 q + 4 k heads of 128 rows rotated, 4 v heads not) with bias, rows
    pair-interleaved by quant.rope_pair_rows; against the oracle's fp64 GEMV on the permuted bytes, un-permuted,
    rotated in fp64 (rotate-half, theta 1e6) and rounded once to bf16; a position 0 call equals the plain GEMV."""
    hd, nq, nkv = 128, 28, 4
    N, K = (nq + 2 * nkv) * hd, 3584
    rope_rows = (nq + nkv) * hd
    ops = make(kind, N, K, seed=31, with_bias=True)
    for name in ("W", "s", "z", "bias"):
        t = getattr(ops, name)
        if t is not None:
            setattr(ops, name, quant.rope_pair_rows(t, rope_rows, hd).contiguous())
    _, lin = ops.oracle(with_bias=True)                    # fp64, permuted row order
    j = np.arange(N)
    nat = j.copy()
    jh = j[:rope_rows] % hd
    nat[:rope_rows] = j[:rope_rows] - jh + (jh >> 1) + (jh & 1) * (hd // 2)
    y_nat = np.empty(N)
    y_nat[nat] = lin                                       # natural order: dimension d of each head at its row
    for pos, theta in ((0.0, 1e6), (1234.0, 1e6), (77.0, 5e5)):
        want = y_nat.copy()
        i = np.arange(hd // 2)
        ang = pos * theta ** (-2.0 * i / hd)
        for h in range(rope_rows // hd):
            a, b = y_nat[h * hd:h * hd + hd // 2], y_nat[h * hd + hd // 2:(h + 1) * hd]
            want[h * hd:h * hd + hd // 2] = a * np.cos(ang) - b * np.sin(ang)
            want[h * hd + hd // 2:(h + 1) * hd] = b * np.cos(ang) + a * np.sin(ang)
        ops.nan_fill()
        p_ = lambda t: None if t is None else t.data_ptr()                 # noqa: E731
        L.rope(kind, p_(ops.W), p_(ops.s), p_(ops.z), ops.x.data_ptr(), ops.bias.data_ptr(), ops.y.data_ptr(), N, K,
               rope_rows, hd, pos, theta)
        torch.cuda.synchronize()
        check(ops, bits(ops.y), O.f64_to_bf16(want), f"rope {kind} pos {pos}")
    assert L.device_error(1) == 0
