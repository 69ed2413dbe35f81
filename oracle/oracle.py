"""CPU oracle for the batch-1 decode GEMV family (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg may import it. It wraps the C restatement in oracle/gemv_oracle.c (formats of Bejaine/PAIA-Project
src/paia_gemv/quant_host.h:18-111 and quant.py:8-38, the asymmetric INT4 convention of
paia-bench/bench/ops/lib_quant.py:159-167 and :223-233) and adds numpy versions of the dequantise-then-matmul
reference (paia-bench/bench/ops/ours_quant.py:69-71) that carry the dot product in fp64 and round once to bf16.

Arrays cross this module as raw bit patterns: bf16 and fp16 tensors are numpy uint16, e4m3 weights and packed
nibbles are uint8, fp32 scales are float32.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "build" / "liboracle.so"
REF_QUANT_PATH = HERE / "_ref" / "libref_quant.so"
REF_CUDA_PATH = HERE / "_ref" / "libpaia_gemv_ref.so"

_lib = None


def build():
    """Compile oracle/gemv_oracle.c into oracle/build/liboracle.so (gcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        for name in ("orc_e4m3_encode_n", "orc_e4m3_decode_n", "orc_f32_to_f16_n", "orc_f16_to_f32_n",
                     "orc_f32_to_bf16_n", "orc_f64_to_bf16_n"):
            getattr(L, name).argtypes = [P, P, S]
            getattr(L, name).restype = None
        L.orc_quantize_fp8_rowwise.argtypes = [P, I, I, P, P]
        L.orc_quantize_int4_g128.argtypes = [P, I, I, P, P]
        L.orc_quantize_int4_asym.argtypes = [P, I, I, P, P, P]
        L.orc_gemv_bf16.argtypes = [P, P, P, I, I, I, I, P, P]
        L.orc_gemv_fp8.argtypes = [P, P, P, P, I, I, I, I, P, P]
        L.orc_gemv_int4.argtypes = [P, P, P, P, I, I, I, I, P, P]
        L.orc_gemv_int4_asym.argtypes = [P, P, P, P, P, I, I, I, I, P, P]
        L.orc_dequant_int4_to_bf16.argtypes = [P, P, I, I, P]
        for name in ("orc_quantize_fp8_rowwise", "orc_quantize_int4_g128", "orc_quantize_int4_asym", "orc_gemv_bf16",
                     "orc_gemv_fp8", "orc_gemv_int4", "orc_gemv_int4_asym", "orc_dequant_int4_to_bf16"):
            getattr(L, name).restype = None
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ------------------------------------------------------------------ element conversions

def _map(fn, a, in_dt, out_dt):
    a = _c(a, in_dt)
    out = np.empty(a.shape, dtype=out_dt)
    getattr(lib(), fn)(_p(a), _p(out), a.size)
    return out


def e4m3_encode(x):
    return _map("orc_e4m3_encode_n", x, np.float32, np.uint8)


def e4m3_decode(b):
    return _map("orc_e4m3_decode_n", b, np.uint8, np.float32)


def f32_to_f16(x):
    return _map("orc_f32_to_f16_n", x, np.float32, np.uint16)


def f16_to_f32(h):
    return _map("orc_f16_to_f32_n", h, np.uint16, np.float32)


def f32_to_bf16(x):
    return _map("orc_f32_to_bf16_n", x, np.float32, np.uint16)


def bf16_to_f32(b):
    return (_c(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f64_to_bf16(x):
    return _map("orc_f64_to_bf16_n", x, np.float64, np.uint16)


_E4M3_LUT = None


def e4m3_lut():
    """float32[256]: the value of every e4m3fn code (NaN for 0x7F and 0xFF)."""
    global _E4M3_LUT
    if _E4M3_LUT is None:
        _E4M3_LUT = e4m3_decode(np.arange(256, dtype=np.uint8))
    return _E4M3_LUT


# ------------------------------------------------------------------ quantisers

def quantize_fp8_rowwise(W):
    """W float32 [N,K] -> (q uint8 [N,K] e4m3 codes, scale float32 [N])."""
    W = _c(W, np.float32)
    N, K = W.shape
    q = np.empty((N, K), dtype=np.uint8)
    s = np.empty(N, dtype=np.float32)
    lib().orc_quantize_fp8_rowwise(_p(W), N, K, _p(q), _p(s))
    return q, s


def quantize_int4_g128(W):
    """W float32 [N,K], K % 128 == 0 -> (packed uint8 [N,K/2], scales fp16 bits uint16 [N,K/128])."""
    W = _c(W, np.float32)
    N, K = W.shape
    assert K % 128 == 0
    p = np.empty((N, K // 2), dtype=np.uint8)
    s = np.empty((N, K // 128), dtype=np.uint16)
    lib().orc_quantize_int4_g128(_p(W), N, K, _p(p), _p(s))
    return p, s


def quantize_int4_asym(W):
    """W float32 [N,K], K % 128 == 0 -> (packed uint8 [N,K/2], scale bf16 bits [N,K/128], zero bf16 bits [N,K/128])."""
    W = _c(W, np.float32)
    N, K = W.shape
    assert K % 128 == 0
    p = np.empty((N, K // 2), dtype=np.uint8)
    s = np.empty((N, K // 128), dtype=np.uint16)
    z = np.empty((N, K // 128), dtype=np.uint16)
    lib().orc_quantize_int4_asym(_p(W), N, K, _p(p), _p(s), _p(z))
    return p, s, z


# ------------------------------------------------------------------ dequantisers (numpy, fp32 like the reference)

def unpack_nibbles(packed):
    """uint8 [N,K/2] -> int32 [N,K] nibbles (byte j: weight 2j in the low nibble, 2j+1 in the high nibble)."""
    p = _c(packed, np.uint8).astype(np.int32)
    N, half = p.shape
    return np.stack([p & 0xF, p >> 4], axis=-1).reshape(N, half * 2)


def dequant_fp8(q, scale):
    return e4m3_lut()[_c(q, np.uint8)] * _c(scale, np.float32)[:, None]


def dequant_int4(packed, scales16):
    n = unpack_nibbles(packed).astype(np.float32) - np.float32(8)
    return n * np.repeat(f16_to_f32(scales16), 128, axis=1)


def dequant_int4_asym(packed, s_bf16, z_bf16):
    n = unpack_nibbles(packed).astype(np.float32) - np.float32(8)
    s = np.repeat(bf16_to_f32(s_bf16), 128, axis=1)
    z = np.repeat(bf16_to_f32(z_bf16), 128, axis=1)
    return (n * s) + z


# ------------------------------------------------------------------ GEMV oracles

def _finish(acc, bias):
    if bias is not None:
        acc = acc + bf16_to_f32(bias).astype(np.float64)
    return f64_to_bf16(acc), acc


def _rows(N, rows):
    return np.arange(N) if rows is None else np.asarray(rows)


def gemv(kind, x, W=None, q=None, scale=None, packed=None, scales=None, zeros=None, bias=None, rows=None,
         chunk=4096):
    """Dequantise-then-matmul in fp64, one rounding to bf16 at the end.

    kind: "bf16" (W bf16 bits [N,K]), "fp8" (q, scale), "int4" (packed, scales fp16 bits), "int4_asym"
    (packed, scales bf16 bits, zeros bf16 bits). x: bf16 bits [K]. bias: bf16 bits [N] or None.
    rows: optional subset of output rows. Returns (y_bf16_bits, y_f64) over the selected rows.
    """
    xd = bf16_to_f32(x).astype(np.float64)
    N = (W if W is not None else (q if q is not None else packed)).shape[0]
    idx = _rows(N, rows)
    outs = []
    for i in range(0, len(idx), chunk):
        r = idx[i:i + chunk]
        if kind == "bf16":
            deq = bf16_to_f32(W[r])
        elif kind == "fp8":
            deq = dequant_fp8(q[r], scale[r])
        elif kind == "int4":
            deq = dequant_int4(packed[r], scales[r])
        elif kind == "int4_asym":
            deq = dequant_int4_asym(packed[r], scales[r], zeros[r])
        else:
            raise ValueError(kind)
        outs.append(deq.astype(np.float64) @ xd)
    acc = np.concatenate(outs) if outs else np.zeros(0)
    return _finish(acc, None if bias is None else _c(bias, np.uint16)[idx])


def gemv_c(kind, x, W=None, q=None, scale=None, packed=None, scales=None, zeros=None, bias=None):
    """The same oracle through the scalar C loops (sequential fp64 sum); used to cross-check gemv() on small cases."""
    L = lib()
    x = _c(x, np.uint16)
    b = None if bias is None else _c(bias, np.uint16)
    if kind == "bf16":
        W = _c(W, np.uint16); N, K = W.shape
    elif kind == "fp8":
        q = _c(q, np.uint8); scale = _c(scale, np.float32); N, K = q.shape
    else:
        packed = _c(packed, np.uint8); scales = _c(scales, np.uint16); N, K = packed.shape[0], packed.shape[1] * 2
    yd = np.empty(N, dtype=np.float64)
    yb = np.empty(N, dtype=np.uint16)
    if kind == "bf16":
        L.orc_gemv_bf16(_p(W), _p(x), _p(b), N, K, 0, N, _p(yd), _p(yb))
    elif kind == "fp8":
        L.orc_gemv_fp8(_p(q), _p(scale), _p(x), _p(b), N, K, 0, N, _p(yd), _p(yb))
    elif kind == "int4":
        L.orc_gemv_int4(_p(packed), _p(scales), _p(x), _p(b), N, K, 0, N, _p(yd), _p(yb))
    elif kind == "int4_asym":
        zeros = _c(zeros, np.uint16)
        L.orc_gemv_int4_asym(_p(packed), _p(scales), _p(zeros), _p(x), _p(b), N, K, 0, N, _p(yd), _p(yb))
    else:
        raise ValueError(kind)
    return yb, yd


def dequant_int4_to_bf16(packed, scales16):
    packed = _c(packed, np.uint8); scales16 = _c(scales16, np.uint16)
    N, K = packed.shape[0], packed.shape[1] * 2
    out = np.empty((N, K), dtype=np.uint16)
    lib().orc_dequant_int4_to_bf16(_p(packed), _p(scales16), N, K, _p(out))
    return out


def silu_mul(gu_bits):
    """bf16(SiLU(gate) * up) of x = [gate | up] (bf16 bits, 2K values), SiLU(v) = v / (1 + e^-v) carried in fp64 and
    rounded once: the activation a fused gate_up projection feeds the down projection."""
    v = bf16_to_f32(_c(gu_bits, np.uint16)).astype(np.float64)
    K = v.shape[0] // 2
    g, u = v[:K], v[K:]
    with np.errstate(over="ignore"):                   # e^-g overflows to inf for g << 0: SiLU -> -0
        return f64_to_bf16(g / (1.0 + np.exp(-g)) * u)


# ------------------------------------------------------------------ comparison metrics

def rel_l2(y_bits, ref_bits):
    """Relative L2 error of bf16 output bits against bf16 reference bits (the parity gate, tolerance 1e-3)."""
    y = bf16_to_f32(y_bits).astype(np.float64)
    r = bf16_to_f32(ref_bits).astype(np.float64)
    d = np.linalg.norm(r)
    return float(np.linalg.norm(y - r) / d) if d > 0 else float(np.linalg.norm(y))


def max_rel(y_bits, ref_f64):
    """The reference harness's own gate: max|y - ref| / max|ref| (< 2e-2), against the unrounded reference."""
    y = bf16_to_f32(y_bits).astype(np.float64)
    d = np.abs(ref_f64).max()
    return float(np.abs(y - ref_f64).max() / d) if d > 0 else float(np.abs(y).max())


# ------------------------------------------------------------------ the reference's own builds (pinning only)

def ref_quant_lib():
    """oracle/_ref/libref_quant.so: the reference's quant_host.h behind a C shim, or None when not built."""
    if not REF_QUANT_PATH.exists():
        return None
    L = ctypes.CDLL(str(REF_QUANT_PATH))
    P, I = ctypes.c_void_p, ctypes.c_int
    L.ref_e4m3_decode.argtypes = [ctypes.c_uint8]; L.ref_e4m3_decode.restype = ctypes.c_float
    L.ref_e4m3_encode.argtypes = [ctypes.c_float]; L.ref_e4m3_encode.restype = ctypes.c_uint8
    L.ref_f32_to_f16.argtypes = [ctypes.c_float]; L.ref_f32_to_f16.restype = ctypes.c_uint16
    L.ref_f16_to_f32.argtypes = [ctypes.c_uint16]; L.ref_f16_to_f32.restype = ctypes.c_float
    L.ref_quantize_fp8_rowwise.argtypes = [P, I, I, P, P]; L.ref_quantize_fp8_rowwise.restype = None
    L.ref_quantize_int4_g128.argtypes = [P, I, I, P, P]; L.ref_quantize_int4_g128.restype = None
    return L


if os.environ.get("PAIA_ORACLE_BUILD_ON_IMPORT") == "1":
    lib()
