"""ctypes loader for libpaia_gemv.so, the B200 (sm_100a) build of the batch-1 decode GEMV family.

Mirrors Bejaine/PAIA-Project src/paia_gemv/loader.py:1-109: the same library search order ($PAIA_GEMV_LIB, then
build/<arch>/, then build/ under the package root), the same `GemvLib` methods with the same arguments (raw device
pointers as ints, launch on torch's current raw CUDA stream so the ops are CUDA-graph capturable), the same variant
tables (`variants`, `variants_fp8`, `variants_int4`: lists of {"id", "R", "U", "W", "S", "H"}) and the same error
behaviour (a nonzero return code raises RuntimeError; -1 bad variant, -2 bad shape or alignment, >0 cudaError_t).

Added for the B200 build: `int4_asym` (asymmetric INT4 g128, bf16 scale and zero), an optional fused bias on every
format (`*_bias`), `variant_info_ex` (the B200 launch configuration a variant maps to), `device_error()`, `layer` and `plan_*` (one
persistent launch for a sequence of GEMVs), and the tensor-parallel helpers used by paia_gemv.tp. There is no CPU fallback: without the library every op raises.
"""
import ctypes
import os
import platform
from pathlib import Path

_PKG_ROOT = Path(__file__).resolve().parent.parent    # paia-project_b200/, the analogue of the reference's src/


def find_lib():
    env = os.environ.get("PAIA_GEMV_LIB")
    cands = [env] if env else []
    cands += [str(_PKG_ROOT / "build" / platform.machine() / "libpaia_gemv.so"),
              str(_PKG_ROOT / "build" / "libpaia_gemv.so")]
    for c in cands:
        if c and os.path.exists(c):
            return c
    raise FileNotFoundError("libpaia_gemv.so not found (run `python paia-project_b200/build.py`, or set "
                            "PAIA_GEMV_LIB). Tried: " + ", ".join(c for c in cands if c))


def current_raw_stream():
    import torch
    return torch._C._cuda_getCurrentRawStream(torch.cuda.current_device())


_KINDS = {"bf16": 0, "fp8": 1, "int4": 2, "int4_asym": 3}
_EX_FIELDS = ("R", "U", "W", "S", "H", "KS", "pdl", "vec_bytes", "math")


class VariantEx(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int) for f in _EX_FIELDS]


class GemvOp(ctypes.Structure):
    """paia_gemv_op: one GEMV of a layer launch (raw device pointers; unused ones None). act = ACT_SILU_MUL: x holds
    [gate | up] (2K values) and the op reads bf16(SiLU(gate) * up)."""
    _fields_ = [("Wq", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("zeros", ctypes.c_void_p),
                ("x", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("N", ctypes.c_int), ("K", ctypes.c_int), ("act", ctypes.c_int)]
    ACT_NONE, ACT_SILU_MUL = 0, 1


MAX_LAYER_OPS = 6


class GemvLib:
    def __init__(self, path=None):
        self.path = path or find_lib()
        lib = ctypes.CDLL(self.path)
        P, I = ctypes.c_void_p, ctypes.c_int
        # --- the reference's C ABI (gemv_bf16.cu:37-53, gemv_quant.cu:59-97), same argtypes as its loader.py:32-46
        lib.paia_gemv_bf16.restype = I
        lib.paia_gemv_bf16.argtypes = [P, P, P, I, I, I, P]
        lib.paia_gemv_bf16_variant_count.restype = I
        lib.paia_gemv_bf16_variant_info.restype = I
        lib.paia_gemv_bf16_variant_info.argtypes = [I] + [ctypes.POINTER(I)] * 5
        lib.paia_gemv_fp8.restype = I
        lib.paia_gemv_fp8.argtypes = [P, P, P, P, I, I, I, P]
        lib.paia_gemv_int4.restype = I
        lib.paia_gemv_int4.argtypes = [P, P, P, P, I, I, I, P]
        lib.paia_gemv_int4_naive.restype = I
        lib.paia_gemv_int4_naive.argtypes = [P, P, P, P, I, I, P]
        lib.paia_gemv_int4_unfused.restype = I
        lib.paia_gemv_int4_unfused.argtypes = [P, P, P, P, P, I, I, P]
        lib.paia_gemv_int4_unfused_static.restype = I
        lib.paia_gemv_int4_unfused_static.argtypes = [P, P, P, P, I, I, P]
        lib.paia_gemv_launch_ex.restype = I
        lib.paia_gemv_launch_ex.argtypes = [I] * 8 + [P] * 6 + [I, I, P]
        lib.paia_gemv_tp.restype = I
        lib.paia_gemv_tp.argtypes = [I, P, P, P, P, P, ctypes.POINTER(P), ctypes.POINTER(P), I, I, I, I, P]
        lib.paia_gemv_tp_ctas.restype = I
        lib.paia_gemv_tp_ctas.argtypes = [I, I, I]
        lib.paia_gemv_tp_deferred.restype = I
        lib.paia_gemv_tp_deferred.argtypes = [I, P, P, P, P, P, ctypes.POINTER(P), ctypes.POINTER(P), I, I, I, I, P]
        lib.paia_gemv_rope.restype = I
        lib.paia_gemv_rope.argtypes = [I, P, P, P, P, P, P, I, I, I, I, ctypes.c_float, ctypes.c_float, P]
        lib.paia_gemv_tp_exchange.restype = I
        lib.paia_gemv_tp_exchange.argtypes = [ctypes.POINTER(P), I, I, P]
        lib.paia_gemv_tp_alloc.restype = I
        lib.paia_gemv_tp_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(P)]
        lib.paia_gemv_tp_free.restype = I
        lib.paia_gemv_tp_free.argtypes = [P]
        lib.paia_gemv_ipc_handle.restype = I
        lib.paia_gemv_ipc_handle.argtypes = [P, ctypes.c_char_p]
        lib.paia_gemv_ipc_open.restype = I
        lib.paia_gemv_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(P)]
        lib.paia_gemv_ipc_close.restype = I
        lib.paia_gemv_ipc_close.argtypes = [P]
        # --- B200 additions
        lib.paia_gemv_batched.restype = I
        lib.paia_gemv_batched.argtypes = [I, P, P, P, P, P, P, I, I, I, P]
        lib.paia_gemv_layer.restype = I
        lib.paia_gemv_layer.argtypes = [I, I, I, ctypes.POINTER(GemvOp), P, P]
        lib.paia_gemv_plan_create.restype = I
        lib.paia_gemv_plan_create.argtypes = [I, I, I, ctypes.POINTER(GemvOp), ctypes.POINTER(P)]
        lib.paia_gemv_plan_launch.restype = I
        lib.paia_gemv_plan_launch.argtypes = [P, P]
        lib.paia_gemv_plan_destroy.restype = I
        lib.paia_gemv_plan_destroy.argtypes = [P]
        lib.paia_gemv_int4_asym.restype = I
        lib.paia_gemv_int4_asym.argtypes = [P, P, P, P, P, I, I, I, P]
        lib.paia_gemv_bf16_bias.restype = I
        lib.paia_gemv_bf16_bias.argtypes = [P, P, P, P, I, I, I, P]
        lib.paia_gemv_fp8_bias.restype = I
        lib.paia_gemv_fp8_bias.argtypes = [P, P, P, P, P, I, I, I, P]
        lib.paia_gemv_int4_bias.restype = I
        lib.paia_gemv_int4_bias.argtypes = [P, P, P, P, P, I, I, I, P]
        lib.paia_gemv_int4_asym_bias.restype = I
        lib.paia_gemv_int4_asym_bias.argtypes = [P, P, P, P, P, P, I, I, I, P]
        lib.paia_gemv_int4_asym_variant_count.restype = I
        lib.paia_gemv_variant_info_ex.restype = I
        lib.paia_gemv_variant_info_ex.argtypes = [I, I, ctypes.POINTER(VariantEx)]
        lib.paia_gemv_device_error.restype = I
        lib.paia_gemv_device_error.argtypes = [I]
        lib.paia_gemv_version.restype = ctypes.c_char_p
        self.variants_fp8 = self._qvariants(lib, "fp8")
        self.variants_int4 = self._qvariants(lib, "int4")
        self._lib = lib
        self._fn = lib.paia_gemv_bf16
        self.n_variants = lib.paia_gemv_bf16_variant_count()
        self.variants = []
        for v in range(self.n_variants):
            R, U, W, S, H = (ctypes.c_int() for _ in range(5))
            assert lib.paia_gemv_bf16_variant_info(v, *map(ctypes.byref, (R, U, W, S, H))) == 0
            self.variants.append({"id": v, "R": R.value, "U": U.value, "W": W.value, "S": S.value, "H": H.value})
        # asymmetric INT4 shares the INT4 variant table (same tuples, same ids)
        self.variants_int4_asym = self.variants_int4
        self.version = lib.paia_gemv_version().decode()

    @staticmethod
    def _qvariants(lib, kind):
        count = getattr(lib, f"paia_gemv_{kind}_variant_count")
        count.restype = ctypes.c_int
        info = getattr(lib, f"paia_gemv_{kind}_variant_info")
        info.restype = ctypes.c_int
        info.argtypes = [ctypes.c_int] + [ctypes.POINTER(ctypes.c_int)] * 4
        out = []
        for v in range(count()):
            R, U, W, H = (ctypes.c_int() for _ in range(4))
            assert info(v, *map(ctypes.byref, (R, U, W, H))) == 0
            out.append({"id": v, "R": R.value, "U": U.value, "W": W.value, "S": 0, "H": H.value})
        return out

    @staticmethod
    def _check(rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed with code {rc} (-1 bad variant, -2 bad shape/alignment, >0 cudaError_t)")

    @staticmethod
    def _st(stream):
        return current_raw_stream() if stream is None else stream

    # ------------------------------------------------------------------ the reference's op API
    def fp8(self, Wq_ptr, scale_ptr, x_ptr, y_ptr, N, K, variant, stream=None):
        """Wq [N,K] e4m3 bytes, scale [N] fp32, x [K] bf16, y [N] bf16; K % 16 == 0."""
        self._check(self._lib.paia_gemv_fp8(Wq_ptr, scale_ptr, x_ptr, y_ptr, N, K, variant, self._st(stream)),
                    "paia_gemv_fp8")

    def int4(self, Wq_ptr, scales_ptr, x_ptr, y_ptr, N, K, variant, stream=None):
        """Wq [N,K/2] packed, scales [N,K/128] fp16; K % 128 == 0. Fused kernel."""
        self._check(self._lib.paia_gemv_int4(Wq_ptr, scales_ptr, x_ptr, y_ptr, N, K, variant, self._st(stream)),
                    "paia_gemv_int4")

    def int4_naive(self, Wq_ptr, scales_ptr, x_ptr, y_ptr, N, K, stream=None):
        self._check(self._lib.paia_gemv_int4_naive(Wq_ptr, scales_ptr, x_ptr, y_ptr, N, K, self._st(stream)),
                    "paia_gemv_int4_naive")

    STATIC_SCRATCH_ELEMS = 16 << 20

    def int4_unfused_static(self, Wq_ptr, scales_ptr, x_ptr, y_ptr, N, K, stream=None):
        """int4_unfused with the library's own 32 MiB scratch, for callers that cannot allocate device memory on the
        call path (a memory pool that owns all of HBM, a host without a device allocator, a loop that must not
        synchronise the device). N * K must not exceed 16 Mi; calls that overlap on the GPU race on the shared
        scratch; the first call on a device looks the scratch's address up, so make it before any stream capture."""
        if N * K > self.STATIC_SCRATCH_ELEMS:
            raise RuntimeError(f"paia_gemv_int4_unfused_static: N*K = {N * K} exceeds the static scratch of "
                               f"{self.STATIC_SCRATCH_ELEMS} elements; use int4_unfused with a caller scratch")
        self._check(self._lib.paia_gemv_int4_unfused_static(Wq_ptr, scales_ptr, x_ptr, y_ptr, N, K, self._st(stream)),
                    "paia_gemv_int4_unfused_static")

    def int4_unfused(self, Wq_ptr, scales_ptr, x_ptr, y_ptr, scratch_ptr, N, K, stream=None):
        self._check(self._lib.paia_gemv_int4_unfused(Wq_ptr, scales_ptr, x_ptr, y_ptr, scratch_ptr, N, K,
                                                     self._st(stream)), "paia_gemv_int4_unfused")

    def bf16(self, W_ptr, x_ptr, y_ptr, N, K, variant, stream=None):
        """y[N] = W[N,K] @ x[K]; pointers are ints. Raises on a nonzero return code."""
        rc = self._fn(W_ptr, x_ptr, y_ptr, N, K, variant, self._st(stream))
        if rc != 0:
            raise RuntimeError(f"paia_gemv_bf16 failed with code {rc} (N={N}, K={K}, variant={variant}); "
                               "-1 bad variant, -2 bad shape/alignment (K%8, 16B pointers), >0 cudaError_t")

    # ------------------------------------------------------------------ B200 additions
    def int4_asym(self, Wq_ptr, scales_ptr, zeros_ptr, x_ptr, y_ptr, N, K, variant, stream=None):
        """Asymmetric INT4 g128: Wq [N,K/2] packed, scales and zeros [N,K/128] bf16; w = (q - 8) * s + z."""
        self._check(self._lib.paia_gemv_int4_asym(Wq_ptr, scales_ptr, zeros_ptr, x_ptr, y_ptr, N, K, variant,
                                                  self._st(stream)), "paia_gemv_int4_asym")

    def bf16_bias(self, W_ptr, x_ptr, bias_ptr, y_ptr, N, K, variant, stream=None):
        self._check(self._lib.paia_gemv_bf16_bias(W_ptr, x_ptr, bias_ptr, y_ptr, N, K, variant, self._st(stream)),
                    "paia_gemv_bf16_bias")

    def fp8_bias(self, Wq_ptr, scale_ptr, x_ptr, bias_ptr, y_ptr, N, K, variant, stream=None):
        self._check(self._lib.paia_gemv_fp8_bias(Wq_ptr, scale_ptr, x_ptr, bias_ptr, y_ptr, N, K, variant,
                                                 self._st(stream)), "paia_gemv_fp8_bias")

    def int4_bias(self, Wq_ptr, scales_ptr, x_ptr, bias_ptr, y_ptr, N, K, variant, stream=None):
        self._check(self._lib.paia_gemv_int4_bias(Wq_ptr, scales_ptr, x_ptr, bias_ptr, y_ptr, N, K, variant,
                                                  self._st(stream)), "paia_gemv_int4_bias")

    def int4_asym_bias(self, Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptr, N, K, variant, stream=None):
        self._check(self._lib.paia_gemv_int4_asym_bias(Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptr, N, K,
                                                       variant, self._st(stream)), "paia_gemv_int4_asym_bias")

    def variant_info_ex(self, kind, v):
        """The B200 launch configuration behind variant v of `kind` ("bf16", "fp8", "int4", "int4_asym")."""
        out = VariantEx()
        self._check(self._lib.paia_gemv_variant_info_ex(_KINDS[kind], v, ctypes.byref(out)), "paia_gemv_variant_info_ex")
        return {f: getattr(out, f) for f in _EX_FIELDS}

    def launch_ex(self, kind, R, U, W, math, pdl, ks, ctas_per_sm, Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr,
                  y_ptr, N, K, stream=None):
        """Any compiled kernel instance (tuning and comparisons): math 0/1 CUDA-core, 2-4 register-fed MMA, 5-8
        TMA-fed MMA (R = ring stages, 0 = auto; ks = shared-memory share | x-first knob << 8 (0 auto, k: k - 1 weight
        stages before the producer waits for the x loads, 255: the whole ring first) | tiled tensor copies << 16)."""
        self._check(self._lib.paia_gemv_launch_ex(_KINDS[kind], R, U, W, math, pdl, ks, ctas_per_sm, Wq_ptr,
                                                  scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptr, N, K,
                                                  self._st(stream)), "paia_gemv_launch_ex")

    # --- row-sharded tensor parallelism (paia_gemv.tp drives these)
    def tp(self, kind, Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptrs, flag_ptrs, world, rank, N_local, K,
           stream=None):
        self._check(self._lib.paia_gemv_tp(_KINDS[kind], Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptrs,
                                           flag_ptrs, world, rank, N_local, K, self._st(stream)), "paia_gemv_tp")

    def tp_deferred(self, kind, Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptrs, flag_ptrs, world, rank,
                    N_local, K, stream=None):
        self._check(self._lib.paia_gemv_tp_deferred(_KINDS[kind], Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr,
                                                    y_ptrs, flag_ptrs, world, rank, N_local, K, self._st(stream)),
                    "paia_gemv_tp_deferred")

    def rope(self, kind, Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptr, N, K, rope_rows, head_dim, pos, theta,
             stream=None):
        """y = RoPE(W x + bias) of a fused QKV projection whose first rope_rows rows are in pair-interleaved order
        (quant.rope_pair_rows); y comes out in the natural order."""
        self._check(self._lib.paia_gemv_rope(_KINDS[kind], Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptr, N, K,
                                             rope_rows, head_dim, float(pos), float(theta), self._st(stream)),
                    "paia_gemv_rope")

    def tp_exchange(self, xflag_ptrs, world, rank, stream=None):
        self._check(self._lib.paia_gemv_tp_exchange(xflag_ptrs, world, rank, self._st(stream)), "paia_gemv_tp_exchange")

    def tp_ctas(self, kind, N_local, K):
        n = self._lib.paia_gemv_tp_ctas(_KINDS[kind], N_local, K)
        if n <= 0:
            raise RuntimeError(f"paia_gemv_tp_ctas failed with code {n} ({kind} {N_local}x{K})")
        return n

    def tp_alloc(self, nbytes):
        p = ctypes.c_void_p()
        self._check(self._lib.paia_gemv_tp_alloc(nbytes, ctypes.byref(p)), "paia_gemv_tp_alloc")
        return p.value

    def tp_free(self, ptr):
        self._check(self._lib.paia_gemv_tp_free(ptr), "paia_gemv_tp_free")

    def ipc_handle(self, ptr):
        buf = ctypes.create_string_buffer(64)
        self._check(self._lib.paia_gemv_ipc_handle(ptr, buf), "paia_gemv_ipc_handle")
        return buf.raw

    def ipc_open(self, handle):
        p = ctypes.c_void_p()
        self._check(self._lib.paia_gemv_ipc_open(bytes(handle), ctypes.byref(p)), "paia_gemv_ipc_open")
        return p.value

    def ipc_close(self, ptr):
        self._check(self._lib.paia_gemv_ipc_close(ptr), "paia_gemv_ipc_close")

    def batched(self, kind, Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptr, M, N, K, stream=None):
        """Y[M, N] = X[M, K] . W^T (+ bias): M activation rows against one weight stream (x, y row-major bf16)."""
        self._check(self._lib.paia_gemv_batched(_KINDS[kind], Wq_ptr, scales_ptr, zeros_ptr, x_ptr, bias_ptr, y_ptr,
                                                 M, N, K, self._st(stream)), "paia_gemv_batched")

    def layer(self, kind, ops, counters_ptr, math=0, stream=None):
        """One launch for a sequence of GEMVs of one format. `ops`: a list of dicts (or GemvOp) with Wq, scales,
        zeros, x, bias, y (raw device pointers or None) and N, K; `counters_ptr`: len(ops) + 1 zeroed uint32 on the
        device (left zero by the kernel)."""
        if not 1 <= len(ops) <= MAX_LAYER_OPS:
            raise ValueError(f"a layer launch takes 1..{MAX_LAYER_OPS} ops, got {len(ops)}")
        arr = (GemvOp * len(ops))(*[o if isinstance(o, GemvOp) else GemvOp(**o) for o in ops])
        self._check(self._lib.paia_gemv_layer(_KINDS[kind], math, len(ops), arr, counters_ptr, self._st(stream)),
                    "paia_gemv_layer")

    def plan_create(self, kind, ops, math=0):
        """A plan for a sequence of up to 4096 GEMVs of one format (ops as for `layer`); returns its handle."""
        arr = (GemvOp * len(ops))(*[o if isinstance(o, GemvOp) else GemvOp(**o) for o in ops])
        h = ctypes.c_void_p()
        self._check(self._lib.paia_gemv_plan_create(_KINDS[kind], math, len(ops), arr, ctypes.byref(h)),
                    "paia_gemv_plan_create")
        return h.value

    def plan_launch(self, plan, stream=None):
        self._check(self._lib.paia_gemv_plan_launch(plan, self._st(stream)), "paia_gemv_plan_launch")

    def plan_destroy(self, plan):
        self._check(self._lib.paia_gemv_plan_destroy(plan), "paia_gemv_plan_destroy")

    def device_error(self, clear=True):
        """The device-side error word (0 = none) written by kernels whose bounded waits gave up."""
        return self._lib.paia_gemv_device_error(1 if clear else 0)


_lib = None


def load_lib():
    global _lib
    if _lib is None:
        _lib = GemvLib()
    return _lib
