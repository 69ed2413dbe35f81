"""Shared helpers of the GPU tests: build operands of every format on the device from seeded inputs, call the product
library through its C ABI (paia_gemv.loader), and compute the CPU oracle on the same bytes."""
import ctypes

import numpy as np
import torch

import oracle as O
from paia_gemv import load_lib, quant, synthetic

KINDS = ("bf16", "fp8", "int4", "int4_asym")
TOL = 1e-3          # relative L2 against the bf16-rounded fp64 oracle
DEFAULT = {"bf16": (2, 4, 4, 0, 1), "fp8": (2, 2, 4, 0, 1), "int4": (4, 2, 4, 0, 1), "int4_asym": (4, 2, 4, 0, 1)}


def bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(a, dtype, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype).to(device)


def variant_id(lib, kind, tup):
    table = {"bf16": lib.variants, "fp8": lib.variants_fp8, "int4": lib.variants_int4,
             "int4_asym": lib.variants_int4_asym}[kind]
    for v in table:
        if (v["R"], v["U"], v["W"], v["S"], v["H"]) == tuple(tup):
            return v["id"]
    raise KeyError(tup)


class Operands:
    """Device operands of one GEMV in one format, plus their CPU bytes for the oracle."""

    def __init__(self, kind, W, x, bias=None):
        self.kind, self.N, self.K = kind, W.shape[0], W.shape[1]
        dev = "cuda"
        self.x = x.to(dev).contiguous()
        self.bias = None if bias is None else bias.to(dev).contiguous()
        self.s = self.z = None
        if kind == "bf16":
            self.W = W.to(torch.bfloat16).to(dev).contiguous()
        elif kind == "fp8":
            self.W, self.s = quant.quantize_fp8_rowwise(W)
        elif kind == "int4":
            self.W, self.s = quant.quantize_int4_g128(W)
        elif kind == "int4_asym":
            self.W, self.s, self.z = quant.quantize_int4_asym(W)
        else:
            raise ValueError(kind)
        self.W = self.W.to(dev).contiguous()
        self.s = None if self.s is None else self.s.to(dev).contiguous()
        self.z = None if self.z is None else self.z.to(dev).contiguous()
        self.y = torch.full((self.N,), float("nan"), device=dev, dtype=torch.bfloat16)

    def nan_fill(self):
        self.y.fill_(float("nan"))

    def call(self, lib, variant, bias=None, stream=None, y=None, x=None):
        """Launch through the C ABI; `bias` (a bf16 device tensor or None) selects the *_bias entry point."""
        y = self.y if y is None else y
        x = self.x if x is None else x
        b = bias
        W, s, z = self.W.data_ptr(), None if self.s is None else self.s.data_ptr(), None if self.z is None else self.z.data_ptr()
        xp, yp, N, K = x.data_ptr(), y.data_ptr(), self.N, self.K
        if b is None:
            if self.kind == "bf16":
                lib.bf16(W, xp, yp, N, K, variant, stream)
            elif self.kind == "fp8":
                lib.fp8(W, s, xp, yp, N, K, variant, stream)
            elif self.kind == "int4":
                lib.int4(W, s, xp, yp, N, K, variant, stream)
            else:
                lib.int4_asym(W, s, z, xp, yp, N, K, variant, stream)
        else:
            bp = b.data_ptr()
            if self.kind == "bf16":
                lib.bf16_bias(W, xp, bp, yp, N, K, variant, stream)
            elif self.kind == "fp8":
                lib.fp8_bias(W, s, xp, bp, yp, N, K, variant, stream)
            elif self.kind == "int4":
                lib.int4_bias(W, s, xp, bp, yp, N, K, variant, stream)
            else:
                lib.int4_asym_bias(W, s, z, xp, bp, yp, N, K, variant, stream)
        return y

    def call_ex(self, lib, R, U, Wn, math, pdl, ks=0, ctas_per_sm=0, with_bias=False):
        kind_id = {"bf16": 0, "fp8": 1, "int4": 2, "int4_asym": 3}[self.kind]
        P = ctypes.c_void_p
        f = lib._lib.paia_gemv_launch_ex
        f.argtypes = [ctypes.c_int] * 8 + [P] * 6 + [ctypes.c_int, ctypes.c_int, P]
        f.restype = ctypes.c_int
        rc = f(kind_id, R, U, Wn, math, pdl, ks, ctas_per_sm, self.W.data_ptr(),
               None if self.s is None else self.s.data_ptr(), None if self.z is None else self.z.data_ptr(),
               self.x.data_ptr(), self.bias.data_ptr() if (with_bias and self.bias is not None) else None,
               self.y.data_ptr(), self.N, self.K, torch.cuda.current_stream().cuda_stream)
        return rc

    def oracle(self, rows=None, with_bias=False, x_bits=None):
        """(bf16 bits, fp64) of the oracle on the same bytes, optionally for a subset of rows."""
        xb = bits(self.x) if x_bits is None else x_bits
        idx = None if rows is None else torch.as_tensor(rows, device="cuda", dtype=torch.long)
        take = (lambda t: t) if idx is None else (lambda t: t.index_select(0, idx))
        b = None
        if with_bias and self.bias is not None:
            b = bits(take(self.bias))
        if self.kind == "bf16":
            return O.gemv("bf16", xb, W=bits(take(self.W)), bias=b)
        if self.kind == "fp8":
            return O.gemv("fp8", xb, q=take(self.W).cpu().numpy(), scale=take(self.s).cpu().numpy(), bias=b)
        if self.kind == "int4":
            return O.gemv("int4", xb, packed=take(self.W).cpu().numpy(), scales=bits(take(self.s)), bias=b)
        return O.gemv("int4_asym", xb, packed=take(self.W).cpu().numpy(), scales=bits(take(self.s)),
                      zeros=bits(take(self.z)), bias=b)


def make(kind, N, K, seed=0, with_bias=False, device="cpu"):
    """Seeded operands (CPU generator by default: identical bytes on every machine)."""
    W, x, b = synthetic.operands(N, K, seed=seed, device=device, with_bias=with_bias)
    return Operands(kind, W, x, b)


def check(ops, y_bits, ref_bits, what=""):
    assert not np.isnan(O.bf16_to_f32(y_bits)).any(), f"{what}: unwritten (NaN) rows"
    err = O.rel_l2(y_bits, ref_bits)
    assert err <= TOL, f"{what}: rel L2 {err:.3e} > {TOL}"
    return err


def lib():
    return load_lib()
