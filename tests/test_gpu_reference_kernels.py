"""GPU: the product kernels against the REFERENCE'S OWN CUDA kernels (Bejaine/PAIA-Project src/paia_gemv/*.cu,
recompiled unmodified for sm_100a into oracle/_ref/libpaia_gemv_ref.so by oracle/Makefile) on identical operands.

Both libraries export the same C ABI, so the same pointers go to both. The outputs must agree within the parity
tolerance (relative L2 <= 1e-3 between the two bf16 outputs) and each must match the oracle. With `-s` the test also
prints graph-mode microseconds of both on the real Llama-3.1-8B / Qwen2.5-7B shapes (L2-rotated operands): this is the
"recompiled reference on the same B200" baseline the B200 kernels are measured against."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from gpu_cases import DEFAULT, bits, check, lib, make, variant_id
from paia_gemv import synthetic, timing

pytestmark = pytest.mark.gpu

REF_DEFAULT = {"bf16": (2, 4, 4, 0, 1), "fp8": (2, 2, 4, 0, 1), "int4": (4, 2, 4, 0, 1)}


def ref_lib():
    if not O.REF_CUDA_PATH.exists():
        pytest.skip("oracle/_ref/libpaia_gemv_ref.so not built")
    from paia_gemv.loader import GemvLib
    return GemvLib.__new__(GemvLib), ctypes.CDLL(str(O.REF_CUDA_PATH))


def ref_call(R, kind, ops, y, variant):
    P, I = ctypes.c_void_p, ctypes.c_int
    st = P(torch.cuda.current_stream().cuda_stream)
    if kind == "bf16":
        R.paia_gemv_bf16.argtypes = [P, P, P, I, I, I, P]
        return R.paia_gemv_bf16(P(ops.W.data_ptr()), P(ops.x.data_ptr()), P(y.data_ptr()), ops.N, ops.K, variant, st)
    fn = R.paia_gemv_fp8 if kind == "fp8" else R.paia_gemv_int4
    fn.argtypes = [P, P, P, P, I, I, I, P]
    return fn(P(ops.W.data_ptr()), P(ops.s.data_ptr()), P(ops.x.data_ptr()), P(y.data_ptr()), ops.N, ops.K, variant, st)


def ref_variant(R, kind, tup):
    I = ctypes.c_int
    if kind == "bf16":
        n = R.paia_gemv_bf16_variant_count()
        for v in range(n):
            a = [I() for _ in range(5)]
            R.paia_gemv_bf16_variant_info(v, *map(ctypes.byref, a))
            if tuple(x.value for x in a) == tup:
                return v
    else:
        cnt = getattr(R, f"paia_gemv_{kind}_variant_count")
        info = getattr(R, f"paia_gemv_{kind}_variant_info")
        for v in range(cnt()):
            a = [I() for _ in range(4)]
            info(v, *map(ctypes.byref, a))
            if (a[0].value, a[1].value, a[2].value, 0, a[3].value) == tup:
                return v
    raise KeyError(tup)


@pytest.mark.parametrize("kind", ["bf16", "fp8", "int4"])
def test_same_results_as_reference_kernels(kind):
    _, R = ref_lib()
    L = lib()
    rv = ref_variant(R, kind, REF_DEFAULT[kind])
    ov = variant_id(L, kind, DEFAULT[kind])
    shapes = [(7, 1024), (1000, 3584), (4096, 4096), (6144, 4096), (3584, 18944)]
    for (N, K) in shapes:
        ops = make(kind, N, K, seed=N ^ K)
        yr = torch.full((N,), float("nan"), device="cuda", dtype=torch.bfloat16)
        assert ref_call(R, kind, ops, yr, rv) == 0
        ops.nan_fill()
        ops.call(L, ov)
        torch.cuda.synchronize()
        ref, _ = ops.oracle()
        check(ops, bits(yr), ref, f"reference kernel {kind} {N}x{K}")
        check(ops, bits(ops.y), ref, f"b200 kernel {kind} {N}x{K}")
        assert O.rel_l2(bits(ops.y), bits(yr)) <= 1e-3


def test_timing_vs_reference_kernels(capsys):
    """Informational timing table (graph mode, L2-rotated). Asserts only that both run."""
    _, R = ref_lib()
    L = lib()
    rows = []
    for kind in ("bf16", "fp8", "int4"):
        rv = ref_variant(R, kind, REF_DEFAULT[kind])
        ov = variant_id(L, kind, DEFAULT[kind])
        for model in ("llama31_8b", "qwen25_7b"):
            for layer in ("qkv_fused", "o_proj", "gate_up_fused", "down_proj"):
                N, K = synthetic.SHAPES[model][layer]
                g = torch.Generator(device="cuda").manual_seed(1)
                base = make(kind, 8, K)          # format template; big operands generated on the device
                wbytes = {"bf16": 2 * N * K, "fp8": N * K + 4 * N, "int4": N * K // 2 + N * K // 64}[kind]
                n = timing.plan_rotation(wbytes)
                copies = []
                for _ in range(n):
                    W = synthetic.weights_f32(N, K, g, device="cuda")
                    x = synthetic.activation_bf16(K, g, device="cuda")
                    from gpu_cases import Operands
                    copies.append(Operands(kind, W, x))
                    del W
                ours = timing.median(timing.time_graph([lambda o=o: o.call(L, ov) for o in copies]))
                refs = timing.median(timing.time_graph(
                    [lambda o=o: ref_call(R, kind, o, o.y, rv) for o in copies]))
                rows.append((kind, model, layer, N, K, wbytes, ours, refs))
                del copies, base
                torch.cuda.empty_cache()
    with capsys.disabled():
        print("\nkind  model       layer          N      K      us(b200)  GB/s    us(ref sm_100a)  GB/s   speedup")
        for kind, model, layer, N, K, wb, o, r in rows:
            print(f"{kind:5s} {model:11s} {layer:14s} {N:6d} {K:6d} {o:9.2f} {wb / o / 1e3:7.0f} {r:12.2f} "
                  f"{wb / r / 1e3:9.0f} {r / o:8.2f}x")
