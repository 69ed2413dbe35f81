"""CPU (no GPU needed): the product library loads, exports every symbol include/paia_gemv.h declares, keeps the
reference's variant-table contract, and rejects bad arguments with the reference's return codes before touching the
device (src/paia_gemv/gemv_bf16.cu:46-51, gemv_quant.cu:65-66, :74-75, :81, :89; pinned on the GPU side by
src/tests/test_gemv_bf16.py:66-71 and gemv_bf16_check.cu:374-376)."""
import ctypes
import importlib.util
import os
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "paia_gemv.h"


def declared_symbols():
    txt = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(paia_gemv_\w+)\s*\(", txt)))


def test_every_declared_symbol_is_exported(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (paia_gemv_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    assert len(declared_symbols()) >= 20


def test_no_torch_dependency(lib_path):
    out = subprocess.run(["ldd", lib_path], capture_output=True, text=True).stdout
    assert "torch" not in out and "c10" not in out and "libcudart.so" not in out   # static cudart, no torch ABI


def test_loader_and_variant_tables(lib_path):
    from paia_gemv import loader
    lib = loader.GemvLib(lib_path)
    # the reference's grids (96 / 36 / 48 tuples, ids as the reference numbers them), then 12 TMA-fed B200 variants
    assert lib.n_variants == 96 + 12 and len(lib.variants_fp8) == 36 + 12 and len(lib.variants_int4) == 48 + 12
    assert len(lib.variants_int4_asym) == 48 + 12
    tup = lambda v: (v["R"], v["U"], v["W"], v["S"], v["H"])
    tma = {(0, U, W, 0, H) for U in (2, 4) for W in (4, 8, 16) for H in (0, 1)}
    for table, n in ((lib.variants, 96), (lib.variants_fp8, 36), (lib.variants_int4, 48), (lib.variants_int4_asym, 48)):
        assert {tup(v) for v in table[n:]} == tma and all(v["R"] > 0 for v in table[:n])
    # the tuples the reference's adapters look up by value (ours_bf16.py:22, ours_quant.py:19)
    assert (2, 4, 4, 0, 1) in {tup(v) for v in lib.variants}
    assert (2, 2, 4, 0, 1) in {tup(v) for v in lib.variants_fp8}
    assert (4, 2, 4, 0, 1) in {tup(v) for v in lib.variants_int4}
    # the whole tuple grid of the reference tables
    assert {tup(v) for v in lib.variants[:96]} == {(R, U, W, S, H) for R in (1, 2, 4) for U in (1, 2, 4, 8)
                                                   for W in (4, 8) for S in (0, 1) for H in (0, 1)}
    assert {tup(v) for v in lib.variants_fp8[:36]} == {(R, U, W, 0, H) for R in (1, 2, 4) for U in (1, 2, 4)
                                                       for W in (4, 8) for H in (0, 1)}
    assert {tup(v) for v in lib.variants_int4[:48]} == {(R, U, W, 0, H) for R in (1, 2, 4, 8) for U in (1, 2, 4)
                                                        for W in (4, 8) for H in (0, 1)}
    ex = lib.variant_info_ex("int4", 0)
    assert ex["vec_bytes"] == 16 and ex["W"] in (4, 8)
    L = lib._lib
    I = ctypes.c_int
    vals = [I() for _ in range(5)]
    assert L.paia_gemv_bf16_variant_info(108, *map(ctypes.byref, vals)) == -1
    assert L.paia_gemv_bf16_variant_info(-1, *map(ctypes.byref, vals)) == -1
    assert "sm_100a" in lib.version


def test_argument_contract_without_gpu(lib_path):
    """Bad variants give -1 and bad shapes/alignments -2, all decided on the host (no device is touched)."""
    L = ctypes.CDLL(lib_path)
    P = ctypes.c_void_p
    a16, a8, a2 = P(0x10000), P(0x10008), P(0x10002)
    for fn in ("paia_gemv_bf16",):
        f = getattr(L, fn)
        f.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        assert f(a16, a16, a16, 4, 16, 108, None) == -1         # variant out of range
        assert f(a16, a16, a16, 4, 16, -1, None) == -1
        assert f(a16, a16, a16, 4, 12, 0, None) == -2           # K % 8
        assert f(a16, a16, a16, 0, 16, 0, None) == -2           # N <= 0
        assert f(a16, a16, a16, 4, 0, 0, None) == -2            # K <= 0
        assert f(a8, a16, a16, 4, 16, 0, None) == -2            # W not 16-byte aligned
        assert f(a16, a8, a16, 4, 16, 0, None) == -2            # x
        assert f(a16, a16, a8, 4, 16, 0, None) == -2            # y
    f = L.paia_gemv_fp8
    f.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
    assert f(a16, a16, a16, a16, 4, 16, 48, None) == -1
    assert f(a16, a16, a16, a16, 4, 24, 0, None) == -2          # K % 16
    assert f(a16, a2, a16, a16, 4, 16, 0, None) == -2           # scale 4-byte alignment
    assert f(a16, a16, a16, P(0x10001), 4, 16, 0, None) == -2   # y 2-byte alignment
    f = L.paia_gemv_int4
    f.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
    assert f(a16, a16, a16, a16, 4, 128, 60, None) == -1
    assert f(a16, a16, a16, a16, 4, 192, 0, None) == -2         # K % 128
    assert f(a16, P(0x10001), a16, a16, 4, 128, 0, None) == -2  # scales 2-byte alignment
    f = L.paia_gemv_int4_naive
    f.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, P]
    assert f(a16, a16, a16, a16, 4, 64, None) == -2
    f = L.paia_gemv_int4_unfused
    f.argtypes = [P, P, P, P, P, ctypes.c_int, ctypes.c_int, P]
    assert f(a16, a16, a16, a16, a8, 4, 128, None) == -2        # scratch 16-byte alignment
    f = L.paia_gemv_int4_asym
    f.argtypes = [P, P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
    assert f(a16, a16, P(0x10001), a16, a16, 4, 128, 0, None) == -2   # zeros 2-byte alignment
    assert f(a16, a16, a16, a16, a16, 4, 128, 60, None) == -1
    f = L.paia_gemv_bf16_bias
    f.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
    assert f(a16, a16, P(0x10001), a16, 4, 16, 0, None) == -2   # bias 2-byte alignment
    f = L.paia_gemv_launch_ex
    f.argtypes = [ctypes.c_int] * 8 + [P] * 6 + [ctypes.c_int, ctypes.c_int, P]
    assert f(2, 3, 1, 8, 1, 1, 0, 0, a16, a16, None, a16, None, a16, 4, 128, None) == -1   # no R=3 instance
    assert f(2, 2, 1, 8, 1, 1, 0, 0, a16, a16, None, a16, None, a16, 4, 100, None) == -2


def _reference_loader():
    from conftest import REFERENCE
    ref = REFERENCE / "src" / "paia_gemv" / "loader.py"
    if not ref.exists():
        pytest.skip("reference checkout not present")
    spec = importlib.util.spec_from_file_location("ref_loader", ref)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_loader_loads_this_library(lib_path, monkeypatch):
    """Drop-in: the reference's own ctypes loader, unmodified, loads this library through $PAIA_GEMV_LIB, declares
    its argtypes and enumerates all three variant tables (its asserts require variant_info == 0 for every id)."""
    mod = _reference_loader()
    monkeypatch.setenv("PAIA_GEMV_LIB", lib_path)
    lib = mod.GemvLib()
    assert lib.path == lib_path and lib.n_variants == 96 + 12
    want = {"R": 2, "U": 4, "W": 4, "S": 0, "H": 1}
    assert any(all(v[k] == want[k] for k in "RUWSH") for v in lib.variants)
    with pytest.raises(RuntimeError):
        lib.bf16(0x10000, 0x10000, 0x10000, 4, 12, 0, stream=0)    # K % 8 -> -2 -> RuntimeError, as the reference


def test_argument_contract_of_the_b200_entry_points(lib_path):
    """The entry points without a reference counterpart reject bad arguments with -2 on the host, before any device
    call: rotary QKV (odd rows or head size, rope rows not whole heads or past N, theta <= 0, pos < 0), tensor
    parallelism (kind, world, rank, missing or misaligned buffers), the exchange, the no-alloc unfused control beyond
    its 16 Mi-element scratch, batched x (M < 1) and layer launches (op count, counters)."""
    L = ctypes.CDLL(lib_path)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    a16 = P(0x10000)
    f = L.paia_gemv_rope
    f.argtypes = [I, P, P, P, P, P, P, I, I, I, I, F, F, P]
    assert f(7, a16, None, None, a16, None, a16, 256, 16, 128, 64, 5.0, 1e4, None) == -2   # kind
    assert f(0, a16, None, None, a16, None, a16, 255, 16, 128, 64, 5.0, 1e4, None) == -2   # odd N
    assert f(0, a16, None, None, a16, None, a16, 256, 16, 128, 63, 5.0, 1e4, None) == -2   # odd head size
    assert f(0, a16, None, None, a16, None, a16, 256, 16, 96, 64, 5.0, 1e4, None) == -2    # rope rows not whole heads
    assert f(0, a16, None, None, a16, None, a16, 256, 16, 320, 64, 5.0, 1e4, None) == -2   # rope rows past N
    assert f(0, a16, None, None, a16, None, a16, 256, 16, 128, 64, 5.0, 0.0, None) == -2   # theta
    assert f(0, a16, None, None, a16, None, a16, 256, 16, 128, 64, -1.0, 1e4, None) == -2  # position
    ptrs = lambda *v: (P * len(v))(*v)                                                      # noqa: E731
    for name in ("paia_gemv_tp", "paia_gemv_tp_deferred"):
        f = getattr(L, name)
        f.argtypes = [I, P, P, P, P, P, ctypes.POINTER(P), ctypes.POINTER(P), I, I, I, I, P]
        y2, fl2 = ptrs(a16, a16), ptrs(a16, a16)
        assert f(5, a16, None, None, a16, None, y2, fl2, 2, 0, 64, 16, None) == -2           # kind
        assert f(0, a16, None, None, a16, None, y2, fl2, 0, 0, 64, 16, None) == -2           # world
        assert f(0, a16, None, None, a16, None, y2, fl2, 9, 0, 64, 16, None) == -2
        assert f(0, a16, None, None, a16, None, y2, fl2, 2, 2, 64, 16, None) == -2           # rank
        assert f(0, a16, None, None, a16, None, None, fl2, 2, 0, 64, 16, None) == -2         # no y pointers
        assert f(0, a16, None, None, a16, None, y2, ptrs(a16, P(0x10004)), 2, 0, 64, 16, None) == -2  # counters
        assert f(0, a16, None, None, a16, None, y2, fl2, 2, 0, 64, 12, None) == -2           # K % 8
    f = L.paia_gemv_tp_exchange
    f.argtypes = [ctypes.POINTER(P), I, I, P]
    assert f(ptrs(a16, a16), 0, 0, None) == -2
    assert f(ptrs(a16, a16), 2, 2, None) == -2
    assert f(None, 2, 0, None) == -2
    assert f(ptrs(a16, P(0x10008)), 2, 0, None) == -2
    f = L.paia_gemv_int4_unfused_static
    f.argtypes = [P, P, P, P, I, I, P]
    assert f(a16, a16, a16, a16, 8192, 4096, None) == -2                                     # past 16 Mi elements
    assert f(a16, a16, a16, a16, 0, 4096, None) == -2
    f = L.paia_gemv_batched
    f.argtypes = [I, P, P, P, P, P, P, I, I, I, P]
    assert f(0, a16, None, None, a16, None, a16, 0, 64, 16, None) == -2                      # M < 1
    assert f(4, a16, None, None, a16, None, a16, 2, 64, 16, None) == -2                      # kind
    f = L.paia_gemv_layer
    f.argtypes = [I, I, I, P, P, P]
    assert f(1, 0, 0, a16, a16, None) == -2                                                  # no ops
    assert f(1, 0, 7, a16, a16, None) == -2                                                  # more than 6
    assert f(1, 0, 2, None, a16, None) == -2                                                 # no op table
    assert f(1, 0, 2, a16, P(0x10002), None) == -2                                           # counters alignment
