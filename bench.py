#!/usr/bin/env python
"""Benchmark of the B200 batch-1 decode GEMV family (the driver's contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}] [--sweep]

Workload (the same at every N: the row-sharded tensor-parallel configuration): one step = the Llama-3.1-8B lm_head
128256x4096 and fused gate_up 28672x4096 in FP8 W8A16 (e4m3 + fp32 row scale) and in INT4 g128 (asymmetric: bf16
scale + bf16 zero), batch 1 -- four GEMVs. On N GPUs (torchrun, one process per GPU) each rank holds N-th of every
matrix's rows and one fused kernel per op stores its outputs into every rank's y over NVLink; on 1 GPU the four
GEMVs run whole (the default path). Weights ~ N(0, 0.02), x ~ N(0, 1) bf16, synthetic; each rank rotates over
copies of its shards so the weights stream from HBM (>= 4 x L2).

value   = full weight bytes (weights + scales / zeros of all four matrices) per step x steps / device time of the K
          steps (CUDA events around a graph replay, max over ranks), GB/s. Strong scaling: the work is fixed.
e2e     = the same metric through the public API (GemvLib methods; ShardedGemv.deferred + TpExchange.run on > 1 GPU)
          with a pinned x copied in and every full y copied out each step, the copies on a second stream overlapping
          the next step's compute (all inside the timed region).
roofline: the dominant kernel (FP8 lm_head rows of the rank): algorithmic bytes / per-launch device time.
cpu_baseline: the reference's CPU path (weights dequantised once, per-call chunked fp32 matmul) on the host cores.
--impl reference: that CPU path alone, as the reference arm (rank 0 only).
Extra keys (1 GPU): the FP8 decode layer (qkv, o, gate_up, down chained), every format's per-shape microseconds on
every Llama / Qwen decode shape, decode microseconds per token.
--sweep, --tp, --families, --decode, --batched, --copy-sweep, --tile-sweep, --one: the studies behind profiles/.
"""
import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "paia-project_b200"))

METRIC = ("GEMV achieved HBM GB/s (weights + scales / device time), Llama-3.1-8B lm_head 128256x4096 + gate_up "
          "28672x4096 in FP8 W8A16 and INT4 g128, batch 1, rows sharded over the GPUs (row-sharded tensor parallel)")
WORKLOAD = ("llama31_8b lm_head 128256x4096 + gate_up_fused 28672x4096, fp8 w8a16 and int4 g128 (asym), batch 1, "
            "row-sharded tensor parallel over n_gpus (1 GPU: whole matrices)")
FALLBACK_HBM_GBS = 6650.0
REASON_BITS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


# ----------------------------------------------------------------------------------------------- helpers

def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def kernel_traffic():
    """dram bytes per launch of the FP8 GEMV kernel from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


class ClockSampler(threading.Thread):
    """NVML sampling of SM clock and clock-event reasons (what `nvidia-smi --query-gpu=clocks.sm,...` reports)."""

    def __init__(self, dev_index, period=0.01):
        super().__init__(daemon=True)
        self.period, self.samples, self.ok = period, [], False
        self._halt = threading.Event()
        self.max_mhz = None
        try:
            import pynvml as N
            import torch
            N.nvmlInit()
            u = str(torch.cuda.get_device_properties(dev_index).uuid)
            u = u if u.startswith("GPU-") else f"GPU-{u}"
            self.h = N.nvmlDeviceGetHandleByUUID(u)
            self.N = N
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self._reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons
            self.ok = True
        except Exception as e:  # NVML missing: report no clocks rather than invent them
            self.err = repr(e)

    def run(self):
        while self.ok and not self._halt.is_set():
            try:
                self.samples.append((time.perf_counter(), self.N.nvmlDeviceGetClockInfo(self.h, self.N.NVML_CLOCK_SM),
                                     int(self._reasons(self.h)),
                                     self.N.nvmlDeviceGetPowerUsage(self.h) / 1000.0))
            except Exception:
                pass
            time.sleep(self.period)

    def stop(self):
        self._halt.set()
        if self.is_alive():
            self.join(timeout=2)

    def summary(self, t0, t1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "NVML unavailable"}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        note = "sampled during the timed region"
        if len(inside) < 3:      # a short timed region: use the samples of the sustained run around it
            inside = [s for s in self.samples if t0 - 1.0 <= s[0] <= t1 + 0.2]
            note = "timed region shorter than the sampling period; samples from the 1 s of load around it"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "note": "no samples"}
        mask = 0
        for s in inside:
            mask |= s[2]
        reasons = [n for b, n in REASON_BITS.items() if mask & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "power_w_max": max(s[3] for s in inside), "samples": len(inside), "note": note}


# ----------------------------------------------------------------------------------------------- operands

class Gemv:
    """One GEMV of a layer: quantised weights on the device, its variant, and a ctypes launch with fixed pointers."""

    def __init__(self, lib, kind, N, K, g, name, bias=False, variant=None, random_codes=False):
        import torch
        from paia_gemv import quant, synthetic
        self.kind, self.N, self.K, self.name = kind, N, K, name
        self.s = self.z = None
        self.bias = synthetic.bias_bf16(N, g, device="cuda") if bias else None
        if random_codes:      # timing-only copies: valid codes of the format, no data-dependent control flow
            if kind == "bf16":
                self.W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
            elif kind == "fp8":
                b = torch.randint(0, 256, (N, K), device="cuda", dtype=torch.uint8, generator=g)
                b[(b & 0x7F) == 0x7F] = 0x7E
                self.W = b
                self.s = torch.rand(N, device="cuda", generator=g) * 1e-4 + 1e-5
            else:
                self.W = torch.randint(0, 256, (N, K // 2), device="cuda", dtype=torch.uint8, generator=g)
                dt = torch.float16 if kind == "int4" else torch.bfloat16
                self.s = (torch.rand(N, K // 128, device="cuda", generator=g) * 1e-3 + 1e-4).to(dt)
                if kind == "int4_asym":
                    self.z = (torch.randn(N, K // 128, device="cuda", generator=g) * 1e-3).to(torch.bfloat16)
        else:
            W = synthetic.weights_f32(N, K, g, device="cuda")
            if kind == "bf16":
                self.W = W.to(torch.bfloat16)
            elif kind == "fp8":
                self.W, self.s = quant.quantize_fp8_rowwise(W)
            elif kind == "int4":
                self.W, self.s = quant.quantize_int4_g128(W)
            else:
                self.W, self.s, self.z = quant.quantize_int4_asym(W)
            del W
        self.variant = variant
        self.lib = lib

    def weight_bytes(self):
        """Algorithmic bytes: weights + scales/zeros (the roofline numerator of the metric)."""
        n = self.W.numel() * self.W.element_size()
        for t in (self.s, self.z):
            if t is not None:
                n += t.numel() * t.element_size()
        return n

    def op_dict(self, x, y):
        p = lambda t: None if t is None else t.data_ptr()      # noqa: E731
        return dict(Wq=p(self.W), scales=p(self.s), zeros=p(self.z), x=p(x), bias=p(self.bias), y=p(y), N=self.N,
                    K=self.K)

    def io_bytes(self):
        return 2 * self.K + 2 * self.N + (2 * self.N if self.bias is not None else 0)

    def launcher(self, x, y):
        """A zero-argument function launching this GEMV on torch's current stream (raw ctypes call)."""
        import ctypes
        import torch
        L = self.lib._lib
        P = ctypes.c_void_p
        W, s, z = P(self.W.data_ptr()), P(self.s.data_ptr() if self.s is not None else 0), \
            P(self.z.data_ptr() if self.z is not None else 0)
        xp, yp = P(x.data_ptr()), P(y.data_ptr())
        b = P(self.bias.data_ptr()) if self.bias is not None else None
        N, K, v = self.N, self.K, self.variant
        dev = torch.cuda.current_device()
        cur = torch._C._cuda_getCurrentRawStream
        if self.kind == "bf16":
            fn = L.paia_gemv_bf16_bias
            return lambda: fn(W, xp, b, yp, N, K, v, P(cur(dev)))
        if self.kind == "fp8":
            fn = L.paia_gemv_fp8_bias
            return lambda: fn(W, s, xp, b, yp, N, K, v, P(cur(dev)))
        if self.kind == "int4":
            fn = L.paia_gemv_int4_bias
            return lambda: fn(W, s, xp, b, yp, N, K, v, P(cur(dev)))
        fn = L.paia_gemv_int4_asym_bias
        return lambda: fn(W, s, z, xp, b, yp, N, K, v, P(cur(dev)))

    def api_call(self, x, y, stream=None):
        """The public op API a user calls (paia_gemv.loader.GemvLib methods); stream None = torch's current one."""
        W, xp, yp, st = self.W.data_ptr(), x.data_ptr(), y.data_ptr(), stream
        if self.kind == "bf16":
            if self.bias is not None:
                return self.lib.bf16_bias(W, xp, self.bias.data_ptr(), yp, self.N, self.K, self.variant, st)
            return self.lib.bf16(W, xp, yp, self.N, self.K, self.variant, st)
        if self.kind == "fp8":
            if self.bias is not None:
                return self.lib.fp8_bias(W, self.s.data_ptr(), xp, self.bias.data_ptr(), yp, self.N, self.K,
                                         self.variant, st)
            return self.lib.fp8(W, self.s.data_ptr(), xp, yp, self.N, self.K, self.variant, st)
        if self.kind == "int4":
            if self.bias is not None:
                return self.lib.int4_bias(W, self.s.data_ptr(), xp, self.bias.data_ptr(), yp, self.N, self.K,
                                          self.variant, st)
            return self.lib.int4(W, self.s.data_ptr(), xp, yp, self.N, self.K, self.variant, st)
        if self.bias is not None:
            return self.lib.int4_asym_bias(W, self.s.data_ptr(), self.z.data_ptr(), xp, self.bias.data_ptr(), yp,
                                           self.N, self.K, self.variant, st)
        return self.lib.int4_asym(W, self.s.data_ptr(), self.z.data_ptr(), xp, yp, self.N, self.K, self.variant, st)


def variant_for(lib, kind, N, K, tuned):
    """Tuned tuple for this shape from paia-project_b200/tuned/b200.json, else the reference adapters' default."""
    defaults = {"bf16": (2, 4, 4, 0, 1), "fp8": (2, 2, 4, 0, 1), "int4": (4, 2, 4, 0, 1), "int4_asym": (4, 2, 4, 0, 1)}
    key = {"bf16": "shapes", "fp8": "fp8_shapes", "int4": "int4_shapes", "int4_asym": "int4_asym_shapes"}[kind]
    want = defaults[kind]
    e = (tuned or {}).get(key, {}).get(f"{N}x{K}")
    if e:
        want = tuple(e["variant"][k] for k in "RUWSH")
    table = {"bf16": lib.variants, "fp8": lib.variants_fp8, "int4": lib.variants_int4,
             "int4_asym": lib.variants_int4_asym}[kind]
    for v in table:
        if (v["R"], v["U"], v["W"], v["S"], v["H"]) == want:
            return v["id"], want
    raise KeyError(want)


def load_tuned():
    p = ROOT / "paia-project_b200" / "tuned" / "b200.json"
    return json.loads(p.read_text()) if p.exists() else None


class Layer:
    """The per-layer GEMV sequence of one decode step, chained: each GEMV reads the previous one's output."""

    def __init__(self, lib, kind, model, g, tuned, random_codes=False):
        import torch
        from paia_gemv import synthetic
        self.gemvs = []
        for name in synthetic.LAYER_SEQUENCE:
            N, K = synthetic.SHAPES[model][name]
            vid, _ = variant_for(lib, kind, N, K, tuned)
            bias = (model == "qwen25_7b" and name == "qkv_fused")
            self.gemvs.append(Gemv(lib, kind, N, K, g, name, bias=bias, variant=vid, random_codes=random_codes))
        self.x = synthetic.activation_bf16(self.gemvs[0].K, g, device="cuda")
        self.ys = [torch.empty(gm.N, dtype=torch.bfloat16, device="cuda") for gm in self.gemvs]
        self.xs = [self.x] + [self.ys[i][:self.gemvs[i + 1].K] for i in range(len(self.gemvs) - 1)]
        self.calls = [gm.launcher(x, y) for gm, x, y in zip(self.gemvs, self.xs, self.ys)]

    def step(self):
        for c in self.calls:
            rc = c()
            if rc:
                raise RuntimeError(f"launch failed with code {rc}")

    def step_api(self, stream=None):
        for gm, x, y in zip(self.gemvs, self.xs, self.ys):
            gm.api_call(x, y, stream)

    def weight_bytes(self):
        return sum(gm.weight_bytes() for gm in self.gemvs)

    def op_dicts(self):
        return [gm.op_dict(x, y) for gm, x, y in zip(self.gemvs, self.xs, self.ys)]

    def layer_launcher(self):
        """A zero-argument function launching this layer's GEMVs as one paia_gemv_layer call (raw ctypes)."""
        import ctypes
        import torch
        from paia_gemv.loader import GemvOp, _KINDS
        ops = (GemvOp * len(self.gemvs))(*[GemvOp(**d) for d in self.op_dicts()])
        self.counters = torch.zeros(len(self.gemvs) + 1, dtype=torch.int32, device="cuda")
        P = ctypes.c_void_p
        fn, kind, n, c = self.gemvs[0].lib._lib.paia_gemv_layer, _KINDS[self.gemvs[0].kind], len(self.gemvs), \
            P(self.counters.data_ptr())
        dev = torch.cuda.current_device()
        cur = torch._C._cuda_getCurrentRawStream
        self._ops = ops
        return lambda: fn(kind, 0, n, ops, c, P(cur(dev)))


def capture(fn, warm=1):
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def check_layer(layer):
    """Sanity check on the device against torch's own fp32 dequantise-then-matmul (not the oracle)."""
    import torch
    from paia_gemv import quant
    layer.step()
    torch.cuda.synchronize()
    errs = []
    for gm, x, y in zip(layer.gemvs, layer.xs, layer.ys):
        if gm.kind == "bf16":
            deq = gm.W.float()
        elif gm.kind == "fp8":
            deq = quant.dequant_fp8(gm.W, gm.s)
        elif gm.kind == "int4":
            deq = quant.dequant_int4(gm.W, gm.s)
        else:
            deq = quant.dequant_int4_asym(gm.W, gm.s, gm.z)
        ref = deq @ x.float()
        if gm.bias is not None:
            ref = ref + gm.bias.float()
        ref = ref.to(torch.bfloat16).float()
        errs.append(((y.float() - ref).norm() / ref.norm()).item())
        del deq
    return max(errs)


# ----------------------------------------------------------------------------------------------- headline workload

# The headline step: Llama-3.1-8B lm_head and fused gate_up in FP8 W8A16 and INT4 g128 (the asymmetric bf16
# scale + zero format), batch 1; rows sharded over the ranks of the launch (one GPU: the whole matrices).
HEADLINE = (("fp8", "lm_head"), ("fp8", "gate_up_fused"), ("int4_asym", "lm_head"), ("int4_asym", "gate_up_fused"))
HEADLINE_MODEL = "llama31_8b"


def format_bytes(kind, N, K):
    """Algorithmic bytes of an N x K weight matrix in a format: weights + scales / zeros (the roofline numerator)."""
    if kind == "bf16":
        return 2 * N * K
    if kind == "fp8":
        return N * K + 4 * N
    if kind == "int4":
        return N * K // 2 + N * K // 64
    return N * K // 2 + N * K // 32


def headline_bytes():
    return sum(format_bytes(k, *synthetic_shape(n)) for k, n in HEADLINE)


def synthetic_shape(name, model=HEADLINE_MODEL):
    from paia_gemv import synthetic
    return synthetic.SHAPES[model][name]


class HeadlineOp:
    """One op of the headline step on this rank: its row shard in `n` L2-rotation copies (copy 0 holds quantised
    weights of this rank's rows, the others valid random codes of the format), and on > 1 GPU the TP objects."""

    def __init__(self, lib, kind, name, world, rank, n, g, bufs=None, exchange=None):
        import torch
        from paia_gemv import tp
        self.kind, self.name = kind, name
        self.N, self.K = synthetic_shape(name)
        r0, r1 = tp.shard_rows(self.N, world, rank)
        self.r0, self.nl = r0, r1 - r0
        self.world = world
        vid, _ = variant_for(lib, kind, self.nl, self.K, load_tuned())
        self.copies = [Gemv(lib, kind, self.nl, self.K, g, name, variant=vid, random_codes=(c > 0)) for c in range(n)]
        self.ys = [torch.empty(self.nl, dtype=torch.bfloat16, device="cuda") for _ in range(n)]
        self.sg = None
        self.exchange = exchange
        if world > 1:
            self.sg = [tp.ShardedGemv(lib, kind, c.W, c.s, c.z, None, self.N, self.K, buffers=bufs) for c in self.copies]

    def shard_bytes(self):
        return self.copies[0].weight_bytes()

    def launcher(self, c, x, deferred=False):
        """Zero-argument launch of copy c: the default-path GEMV (1 GPU), or the TP call: complete (y whole on every
        rank when it ends) or deferred (y whole after the step's exchange)."""
        if self.sg is None:
            return self.copies[c].launcher(x, self.ys[c])
        sg, ex = self.sg[c], self.exchange

        def call():
            if deferred:
                sg.deferred(x)             # raises on a nonzero return code
            else:
                sg.fused(x)
            return 0
        return call

    def output(self, c):
        return self.ys[c] if self.sg is None else self.sg[c].y

    def api_call(self, c, x, stream=None):
        """The public API call a user makes for copy c (GemvLib method, or ShardedGemv.deferred; the step's
        exchange completes the outputs)."""
        if self.sg is None:
            self.copies[c].api_call(x, self.ys[c], stream)
            return self.ys[c]
        return self.sg[c].deferred(x, stream)


def torch_reference(gm, x):
    """fp32 dequantise-then-matmul on the device with torch (the sanity check; the CPU oracle is test-only)."""
    from paia_gemv import quant
    if gm.kind == "bf16":
        deq = gm.W.float()
    elif gm.kind == "fp8":
        deq = quant.dequant_fp8(gm.W, gm.s)
    elif gm.kind == "int4":
        deq = quant.dequant_int4(gm.W, gm.s)
    else:
        deq = quant.dequant_int4_asym(gm.W, gm.s, gm.z)
    ref = deq @ x.float()
    if gm.bias is not None:
        ref = ref + gm.bias.float()
    return ref


def check_headline(ops, x, world):
    """Before timing, on every rank: each op's rows of this rank against torch fp32 (rel L2 <= 1e-3 after bf16
    rounding), and on > 1 GPU the fused peer-store y equal bit for bit to the NCCL all-gather y (which proves the
    exchange). Returns (worst rel L2, all fused == NCCL)."""
    import torch
    worst, same = 0.0, True
    for op in ops:
        gm = op.copies[0]
        op.launcher(0, x)()
        torch.cuda.synchronize()
        y = op.output(0)
        mine = y if world == 1 else y[op.r0:op.r0 + op.nl]
        ref = torch_reference(gm, x).to(torch.bfloat16).float()
        worst = max(worst, ((mine.float() - ref).norm() / ref.norm()).item())
        if world > 1:
            yf = y.clone()
            yn = op.sg[0].nccl(x).clone()
            y.zero_()
            torch.cuda.synchronize()
            import torch.distributed as dist
            dist.barrier()
            op.launcher(0, x, deferred=True)()
            op.exchange.run()
            torch.cuda.synchronize()
            yd = y.clone()
            same = (same and bool(torch.equal(yf.view(torch.int16), yn.view(torch.int16)))
                    and bool(torch.equal(yf.view(torch.int16), yd.view(torch.int16))))
    return worst, same


def time_ops_graph(calls_per_step, steps_per_replay, samples=10, warmup=3):
    """Device microseconds per step of a CUDA graph holding `steps_per_replay` steps (each a list of launches),
    CUDA events on the capturing stream; the same count of launches on every rank."""
    import torch

    def fn():
        for i in range(steps_per_replay):
            for c in calls_per_step[i % len(calls_per_step)]:
                rc = c()
                if rc:
                    raise RuntimeError(f"launch failed with code {rc}")
    gph = capture(fn)
    for _ in range(warmup):
        gph.replay()
    torch.cuda.synchronize()
    out = []
    for _ in range(samples):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gph.replay()
        e1.record()
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1) * 1e3 / steps_per_replay)
    del gph
    return statistics.median(out)


def max_over_ranks(vals, world):
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


# ----------------------------------------------------------------------------------------------- CPU baseline

def cpu_headline_operands(frac, seed=0):
    """Seeded CPU operands of the headline step, the first `frac` of every op's rows (a bounded sample of the same
    workload): (kind, rows, K, W, s, z, x) per op."""
    import torch
    from paia_gemv import quant, synthetic
    g = synthetic.generator(seed)
    ops = []
    for kind, name in HEADLINE:
        N, K = synthetic_shape(name)
        rows = max(1, int(round(N * frac)))
        W = synthetic.weights_f32(rows, K, g)
        x = synthetic.activation_bf16(K, g)
        if kind == "fp8":
            q, s = quant.quantize_fp8_rowwise(W)
            ops.append((kind, rows, K, q, s, None, x))
        else:
            p_, s, z = quant.quantize_int4_asym(W)
            ops.append((kind, rows, K, p_, s, z, x))
        del W
    return ops


def cpu_prepare(ops):
    """The reference op's build step: dequantise every sampled op once (ours_quant.py:99, :138). Returns
    ([(x, Wdeq)], algorithmic bytes of the sample, seconds spent dequantising)."""
    import cpu_reference as C
    prepared, nbytes = [], 0
    t0 = time.perf_counter()
    for (kind, rows, K, W, s, z, x) in ops:
        prepared.append((x, C.dequant(kind, W, s, z)))
        nbytes += format_bytes(kind, rows, K)
    return prepared, nbytes, time.perf_counter() - t0


def cpu_step(prepared):
    """The reference's per-call CPU work for every sampled op: the chunked fp32 matmul (ours_quant.py:69-71)."""
    import cpu_reference as C
    for x, deq in prepared:
        C.matmul(x, deq)


def cpu_calibrate(target_step_s):
    """Row fraction whose per-step matmul takes about target_step_s on this host (measured on a 1/16 sample)."""
    probe = 1.0 / 16
    prepared, _, _ = cpu_prepare(cpu_headline_operands(probe))
    cpu_step(prepared)
    t0 = time.perf_counter()
    cpu_step(prepared)
    t = max(time.perf_counter() - t0, 1e-4)
    return max(1e-3, min(1.0, probe * target_step_s / t))


def cpu_baseline(target_s=15.0):
    """The reference's CPU path for the headline workload on this host's cores: weights dequantised once (reported
    apart), then the timed per-call chunked fp32 matmul over a bounded row sample, median of many reps."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_reference as C
    threads = C.set_threads()
    frac = cpu_calibrate(0.05)
    prepared, nbytes, t_deq = cpu_prepare(cpu_headline_operands(frac))
    cpu_step(prepared)
    t0 = time.perf_counter()
    cpu_step(prepared)
    t1 = max(time.perf_counter() - t0, 1e-4)
    reps = max(10, min(2000, int(target_s / t1)))
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        cpu_step(prepared)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": nbytes / med / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": (f"{frac:.4f} of the rows of each headline op (Llama-3.1-8B lm_head and gate_up in FP8 and INT4 "
                       f"asym; {nbytes / 2**20:.1f} MiB of format bytes): per call the chunked fp32 matmul over "
                       f"weights dequantised once, as the reference op's check (paia-bench ours_quant.py:69-71 over "
                       f"the dequantisation of :99, :138); median of {reps} reps after 1 warm-up; CPU {C.cpu_model()},"
                       f" torch threads {threads}, os.cpu_count {os.cpu_count()}"),
            "dequant_s_once": round(t_deq, 4)}


# ----------------------------------------------------------------------------------------------- arms

def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU implementation of the headline workload on this host's cores (weights
    dequantised once, then the per-call chunked fp32 matmul), rank 0 only; the other ranks exit without work."""
    if rank != 0:
        return 0
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_reference as C
    threads = C.set_threads()
    budget = 120.0
    frac = cpu_calibrate(budget / max(1, args.steps + args.warmup))
    prepared, nbytes, t_deq = cpu_prepare(cpu_headline_operands(frac))
    for _ in range(args.warmup):
        cpu_step(prepared)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(prepared)
    dt = time.perf_counter() - t0
    value = nbytes * args.steps / dt / 1e9
    sample = (f"each step: {frac:.4f} of the rows of every headline op (Llama-3.1-8B lm_head and gate_up in FP8 and "
              f"INT4 asym; {nbytes / 2**20:.2f} MiB of format bytes), the chunked fp32 matmul over weights "
              f"dequantised once (dequantisation {t_deq * 1e3:.0f} ms, untimed, as the reference op does it at build "
              f"time); the reference harness's CPU path restated in oracle/cpu_reference.py; CPU {C.cpu_model()}, "
              f"{threads} torch threads")
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantised to e4m3 / asymmetric int4 g128, N(0,1) bf16 x)",
            "config": {"workload": WORKLOAD, "device": "cpu"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_main(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from paia_gemv import load_lib, synthetic, timing, tp
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    lib = load_lib()
    g = torch.Generator(device="cuda").manual_seed(1000 * rank + 1)
    l2 = timing.l2_bytes()
    # per-rank bytes of one step (this rank's shards), and L2 rotation over n copies of every shard
    step_shard = sum(format_bytes(k, synthetic_shape(n)[0] // world, synthetic_shape(n)[1]) for k, n in HEADLINE)
    n = timing.plan_rotation(step_shard, l2)
    # > 1 GPU: every op its own output buffers (a deferred call per buffer set between two exchanges), one exchange
    bufs, exchange = [], None
    if world > 1:
        exchange = tp.TpExchange(lib, torch.device("cuda", local_rank))
        bufs = [tp.TpBuffers(lib, synthetic_shape(name)[0], torch.device("cuda", local_rank)) for _, name in HEADLINE]
    ops = [HeadlineOp(lib, kind, name, world, rank, n, g, bufs[i] if bufs else None, exchange)
           for i, (kind, name) in enumerate(HEADLINE)]
    gx = torch.Generator(device="cuda").manual_seed(7)                # x is the same on every rank
    x = torch.randn(ops[0].K, device="cuda", generator=gx).to(torch.bfloat16)
    check_err, same = check_headline(ops, x, world)
    bad = max_over_ranks([0.0 if (check_err <= 1e-3 and same) else 1.0, check_err], world)
    if bad[0]:
        raise RuntimeError(f"headline check failed on some rank: worst rel L2 {bad[1]:.3e} against torch fp32, "
                           f"fused == NCCL on this rank: {same}")
    lib.device_error(1)

    def exchange_call():
        exchange.run()
        return 0
    steps_calls = [[op.launcher(c, x, deferred=world > 1) for op in ops] + ([exchange_call] if world > 1 else [])
                   for c in range(n)]

    def run_steps(k):
        for i in range(k):
            for c in steps_calls[i % n]:
                rc = c()
                if rc:
                    raise RuntimeError(f"launch failed with code {rc}")

    # graphs: one full rotation (n steps) and the tails, so exactly K (or W) steps run, the same on every rank
    g_round = capture(lambda: run_steps(n))
    tails = {}
    for k in {args.steps % n, args.warmup % n} - {0}:
        tails[k] = capture(lambda k=k: run_steps(k))

    def replay(k):
        for _ in range(k // n):
            g_round.replay()
        if k % n:
            tails[k % n].replay()

    sampler = ClockSampler(local_rank)
    sampler.start()
    replay(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_host0 = time.perf_counter()
    e0.record()
    replay(args.steps)
    e1.record()
    torch.cuda.synchronize()
    t_host1 = time.perf_counter()
    sampler.stop()
    clocks = sampler.summary(t_host0, t_host1)
    ms = e0.elapsed_time(e1)
    err = lib.device_error(1)
    ms_max, err_max = max_over_ranks([ms, float(err)], world)
    if err_max:
        raise RuntimeError(f"device error {int(err_max)} during the timed steps")
    del g_round, tails
    total_bytes = headline_bytes() * args.steps
    value = total_bytes / (ms_max * 1e-3) / 1e9
    launches = (len(HEADLINE) + (1 if world > 1 else 0)) * args.steps * world

    # per-op device time inside the same kind of graph (every rank the same launches), max over ranks
    reps = max(n, (32 // n) * n)
    per_op = {}
    for op in ops:
        us = time_ops_graph([[op.launcher(c, x)] for c in range(n)], reps)
        per_op[f"{op.kind}:{op.name}"] = us
    keys = list(per_op)
    per_op = dict(zip(keys, max_over_ranks([per_op[k] for k in keys], world)))

    # NCCL all-gather baseline of the same step (> 1 GPU): the same kernel into the local slice, then
    # all_gather_into_tensor, eager, max over ranks
    nccl = None
    if world > 1:
        def nccl_step(i):
            for op in ops:
                op.sg[i % n].nccl(x)
        for i in range(2 * n):
            nccl_step(i)
        torch.cuda.synchronize()
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for i in range(reps):
            nccl_step(i)
        a1.record()
        torch.cuda.synchronize()
        nccl_us = max_over_ranks([a0.elapsed_time(a1) * 1e3 / reps], world)[0]
        nccl = {"us_per_step": round(nccl_us, 3), "GBps": round(headline_bytes() / nccl_us / 1e3, 1),
                "how": "per op: the same TMA kernel into the local slice, then torch.distributed "
                       "all_gather_into_tensor (NCCL) on the compute stream, eager launches, max over ranks"}

    # e2e through the public API with host buffers: every step x copied in from pinned memory, the four ops called
    # eagerly through the user-facing API (GemvLib methods; ShardedGemv.deferred + TpExchange.run on > 1 GPU), every
    # op's full y copied out to pinned memory; CUDA events, max over ranks. The copies run on a second stream, as a
    # user overlaps them: step i's outputs go to the host while step i + 1 computes (its ops write the other rotation
    # copy's y), and x of step i + n is copied in once step i's ops have read x_dev[i mod n]. Every copy of every
    # timed step completes inside the timed region.
    x_host = torch.empty(x.numel(), dtype=torch.bfloat16).pin_memory()
    x_host.copy_(x.cpu())
    y_host = [[torch.empty(op.N, dtype=torch.bfloat16).pin_memory() for op in ops] for _ in range(n)]
    x_dev = [torch.empty_like(x) for _ in range(n)]
    comp, cs = torch.cuda.current_stream(), torch.cuda.Stream()
    ev_x = [torch.cuda.Event() for _ in range(n)]          # on cs: x_dev[c] loaded (and copy c's last outputs out)
    ev_done = [torch.cuda.Event() for _ in range(n)]       # on comp: the ops of the step that used copy c are done

    def load_x(c):
        with torch.cuda.stream(cs):
            x_dev[c].copy_(x_host, non_blocking=True)
            ev_x[c].record(cs)

    def e2e_step(i):
        c = i % n
        comp.wait_event(ev_x[c])                           # x in, and the previous outputs of copy c out
        ys = [op.api_call(c, x_dev[c]) for op in ops]
        if exchange is not None:
            exchange.run()
        ev_done[c].record(comp)
        with torch.cuda.stream(cs):
            cs.wait_event(ev_done[c])
            for y, yh in zip(ys, y_host[c]):
                yh.copy_(y, non_blocking=True)
        load_x(c)                                          # x of step i + n

    for c in range(n):
        load_x(c)
    for i in range(max(3, args.warmup // 10)):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_steps = max(n, min(args.steps, 200))
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(comp)
    cs.wait_event(b0)
    for c in range(n):
        load_x(c)
    for i in range(e2e_steps):
        e2e_step(i)
    comp.wait_stream(cs)
    b1.record(comp)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks([b0.elapsed_time(b1)], world)[0]
    if not all(bool(torch.isfinite(yh.float()).all()) for yc in y_host for yh in yc):
        raise RuntimeError("e2e: non-finite output copied to the host")
    e2e_value = headline_bytes() * e2e_steps / (e2e_ms * 1e-3) / 1e9

    # the same steps with every copy in stream order on the compute stream (no overlap), reported beside it
    def serial_step(i):
        c = i % n
        x_dev[c].copy_(x_host, non_blocking=True)
        ys = [op.api_call(c, x_dev[c]) for op in ops]
        if exchange is not None:
            exchange.run()
        for y, yh in zip(ys, y_host[c]):
            yh.copy_(y, non_blocking=True)

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(comp)
    for i in range(e2e_steps):
        serial_step(i)
    s1.record(comp)
    torch.cuda.synchronize()
    serial_ms = max_over_ranks([s0.elapsed_time(s1)], world)[0]
    e2e_serial = headline_bytes() * e2e_steps / (serial_ms * 1e-3) / 1e9

    # roofline of the dominant kernel: FP8 lm_head (this rank's shard), bytes per launch / per-launch device time
    peak, peak_src = measured_peaks()
    dom = ops[0]
    dom_us = per_op[f"{dom.kind}:{dom.name}"]
    dom_bytes = dom.shard_bytes()
    achieved = dom_bytes / (dom_us * 1e-6) / 1e9
    traffic = kernel_traffic()
    tr = (traffic or {}).get("fp8_lm_head_dram_bytes_per_launch")
    tr_ranks = (traffic or {}).get("fp8_lm_head_rows")

    extras = {}
    if world == 1 and not args.no_extras:
        del steps_calls
        for op in ops:
            op.copies = op.ys = None
        torch.cuda.empty_cache()
        extras = run_extras(lib, g, l2, peak, args)

    result = None
    if rank == 0:
        cb = None
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_baseline()
            cb = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in cb.items()}
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 accumulate (fp8 e4m3 / int4 weights x bf16 x on the tensor cores)",
            "data": "synthetic (seeded N(0,0.02) weights quantised to e4m3 + fp32 row scale and to asymmetric int4 "
                    "g128 with bf16 scale + zero, N(0,1) bf16 x)",
            "config": {"workload": WORKLOAD, "rows_per_rank": {f"{op.kind}:{op.name}": op.nl for op in ops},
                       "rotation_copies": n, "bytes_per_step_all_ranks": headline_bytes(),
                       "l2": f"inputs larger than L2: each rank rotates over {n} copies of its shards = "
                             f"{n * step_shard / 2**20:.0f} MiB >= 4 x L2 ({l2 / 2**20:.0f} MiB)",
                       "launch": ("CUDA graph of back-to-back launches with programmatic dependent launch"
                                  + ("; each op one TMA kernel per rank storing its outputs into every rank's y over "
                                     "NVLink (deferred form, after a per-buffer start handshake), then one exchange "
                                     "kernel per step (system fence, per-rank counts, bounded wait) after which "
                                     "every op's full y is complete on every rank" if world > 1 else "")),
                       "parallelism": f"row-sharded tensor parallel x{world}" if world > 1 else "1 GPU"},
            "per_op_us": {k: round(v, 3) for k, v in per_op.items()},
            "us_per_step": round(ms_max * 1e3 / args.steps, 3),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src + " (burst copy)",
                         "traffic": (round(tr * dom.nl / tr_ranks) if tr and tr_ranks else None),
                         "traffic_source": ("dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of "
                                            "this kernel (profiles/traffic.json), scaled by rows" if tr else None),
                         "algorithmic_bytes_per_launch": dom_bytes,
                         "kernel": f"pb2::gemv_tma_kernel<FP8, 8, 2, 3> ({dom.name} {dom.nl}x{dom.K} rows of this "
                                   f"rank: e4m3 weights + fp32 row scales; per-launch time from CUDA events over a "
                                   f"graph of rotated launches{', including the exchange' if world > 1 else ''})"},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": x.numel() * 2,
                    "d2h_bytes_per_step": sum(op.N * 2 for op in ops), "steps": e2e_steps,
                    "value_copies_in_stream_order": round(e2e_serial, 2),
                    "how": "public API (paia_gemv.loader GemvLib methods; on > 1 GPU tp.ShardedGemv.deferred and "
                           "TpExchange.run), eager launches; per step a pinned H2D of x and a pinned D2H of every op's "
                           "full y on a copy stream (step i's outputs leave while step i + 1 computes into the other "
                           "rotation copy's buffers), the ops on the compute stream; CUDA events around all steps "
                           "and all their copies, max over ranks"},
            "gpu_launches": launches,
            "clocks": clocks,
            "check_rel_l2_vs_torch": round(bad[1], 7),
        }
        if world > 1:
            result["fused_equals_nccl_bitwise"] = True
            result["nccl_all_gather"] = nccl
        result.update(extras)
        if cb is not None:
            result["cpu_baseline"] = cb
    if world > 1:
        dist.barrier()
        for op in ops:
            op.sg = None
        for b in bufs:
            b.close()
        exchange.close()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)
    return 0


def run_extras(lib, g, l2, peak, args):
    """1-GPU extra keys of the bench line: the FP8 decode layer (the previous headline), every format's per-shape
    microseconds on every Llama-3.1-8B and Qwen2.5-7B decode shape, and decode microseconds per token."""
    import torch
    from paia_gemv import synthetic, timing
    out = {}
    # the Llama-3.1-8B FP8 decode layer: qkv -> o -> gate_up -> down chained, rotated over >= 4 x L2 of layers
    tuned = load_tuned()
    probe = Layer(lib, "fp8", "llama31_8b", g, tuned)
    lbytes = probe.weight_bytes()
    L = max(4, math.ceil(4 * l2 / lbytes))
    layers = [probe] + [Layer(lib, "fp8", "llama31_8b", g, tuned, random_codes=True) for _ in range(L - 1)]
    us_layer = time_ops_graph([lay.calls for lay in layers], L * max(1, 40 // L))
    out["decode_layer_fp8"] = {"us_per_layer": round(us_layer, 3), "GBps": round(lbytes / us_layer / 1e3, 1),
                               "frac_of_peak": round(lbytes / us_layer / 1e3 / peak, 4),
                               "how": "Llama-3.1-8B FP8 qkv -> o -> gate_up -> down, each reading the previous "
                                      "output, CUDA graph with PDL, rotated over " + str(L) + " layers"}
    del layers, probe
    torch.cuda.empty_cache()
    shapes = {}
    for kind in ("bf16", "fp8", "int4", "int4_asym"):
        for model in ("llama31_8b", "qwen25_7b"):
            for name in ("qkv_fused", "o_proj", "gate_up_fused", "down_proj", "lm_head"):
                N, K = synthetic.SHAPES[model][name]
                vid, tup = variant_for(lib, kind, N, K, tuned)
                bias = model == "qwen25_7b" and name == "qkv_fused"
                first = Gemv(lib, kind, N, K, g, name, bias=bias, variant=vid, random_codes=True)
                nc = timing.plan_rotation(first.weight_bytes(), l2)
                copies = [first] + [Gemv(lib, kind, N, K, g, name, bias=bias, variant=vid, random_codes=True)
                                    for _ in range(nc - 1)]
                xs = [torch.randn(K, device="cuda", generator=g).to(torch.bfloat16) for _ in copies]
                ys = [torch.empty(N, device="cuda", dtype=torch.bfloat16) for _ in copies]
                calls = [c.launcher(xx, yy) for c, xx, yy in zip(copies, xs, ys)]
                us = timing.median(timing.time_graph(calls, samples=9))
                wb = first.weight_bytes()
                shapes[f"{kind}:{model}:{name}"] = {"N": N, "K": K, "variant": tup, "us": round(us, 3),
                                                    "GBps": round(wb / us / 1e3, 1),
                                                    "frac": round(wb / us / 1e3 / peak, 4)}
                del copies, xs, ys, calls, first
                torch.cuda.empty_cache()
    out["per_shape_us"] = shapes
    tokens, plans = {}, {}
    for kind in ("bf16", "fp8", "int4", "int4_asym"):
        for model in ("llama31_8b", "qwen25_7b"):
            d = decode_token(lib, kind, model, g, tuned, peak, "per_op", reps=5)
            tokens[f"{kind}:{model}"] = {"us_per_token": d["decode_us_per_token"], "GBps": d["GBps"],
                                         "frac": d["frac_of_peak"]}
            if kind.startswith("int4"):                  # the whole token as one plan launch: INT4's faster form
                d = decode_token(lib, kind, model, g, tuned, peak, "plan", reps=5)
                plans[f"{kind}:{model}"] = {"us_per_token": d["decode_us_per_token"], "GBps": d["GBps"],
                                            "frac": d["frac_of_peak"]}
    out["decode_us_per_token"] = tokens
    out["decode_how"] = ("per token: every layer's qkv, o, gate_up, down chained (distinct weights per layer, Qwen qkv "
                         "with bias), then the lm_head; one CUDA graph with PDL (the reference's per-token sum of "
                         "per-op launches, paia-bench analyze_e4.py:177-196, measured as one sequence)")
    out["decode_us_per_token_plan"] = plans
    out["decode_plan_how"] = ("the same token as one paia_gemv_plan launch (every GEMV of the token in one persistent "
                              "kernel, the next op's weights streaming while the previous op finishes), INT4 formats")
    return out


def run_sweep(args):
    """Every Llama and Qwen decode shape in every format (graph mode, L2 rotation), one JSON line each, plus the decode
    us/token of both models in every format (layers back to back with PDL, distinct weights per layer)."""
    import torch
    from paia_gemv import load_lib, synthetic, timing
    torch.cuda.set_device(0)
    lib = load_lib()
    tuned = load_tuned()
    peak, src = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(7)
    l2 = timing.l2_bytes()
    kinds = args.kinds.split(",")
    for kind in kinds:
        for model in ("llama31_8b", "qwen25_7b"):
            for name in ("qkv_fused", "o_proj", "gate_up_fused", "down_proj", "lm_head", "q_proj", "k_proj",
                         "gate_proj"):
                N, K = synthetic.SHAPES[model][name]
                vid, tup = variant_for(lib, kind, N, K, tuned)
                bias = model == "qwen25_7b" and name == "qkv_fused"
                first = Gemv(lib, kind, N, K, g, name, bias=bias, variant=vid)
                n = timing.plan_rotation(first.weight_bytes(), l2)
                copies = [first] + [Gemv(lib, kind, N, K, g, name, bias=bias, variant=vid, random_codes=True)
                                    for _ in range(n - 1)]
                xs = [torch.randn(K, device="cuda", generator=g).to(torch.bfloat16) for _ in copies]
                ys = [torch.empty(N, device="cuda", dtype=torch.bfloat16) for _ in copies]
                calls = [c.launcher(x, y) for c, x, y in zip(copies, xs, ys)]
                us = timing.median(timing.time_graph(calls, samples=15))
                wb = first.weight_bytes()
                print(json.dumps({"kind": kind, "model": model, "layer": name, "N": N, "K": K, "variant": tup,
                                  "us": round(us, 3), "GBps": round(wb / us / 1e3, 1),
                                  "frac_of_peak": round(wb / us / 1e3 / peak, 4), "peak": peak, "peak_source": src,
                                  "copies": n}), flush=True)
                del copies, xs, ys, calls, first
                torch.cuda.empty_cache()
        for model in ("llama31_8b", "qwen25_7b"):
            print(json.dumps(decode_token(lib, kind, model, g, tuned, peak, "per_op")), flush=True)
    return 0


def decode_token(lib, kind, model, g, tuned, peak, mode, reps=10):
    """µs per token of a model's decode GEMVs (every layer's qkv, o, gate_up, down, chained, then the lm_head; distinct
    weights per layer), timed as a CUDA graph. mode "per_op": one launch per GEMV with programmatic dependent launch
    (the reference's per-token sum of per-op launches); "layer": one paia_gemv_layer launch per layer, then the
    lm_head; "plan": one paia_gemv_plan launch for the whole token."""
    import torch
    from paia_gemv import synthetic
    from paia_gemv.loader import GemvOp
    nl = synthetic.N_LAYERS[model]
    layers = [Layer(lib, kind, model, g, tuned, random_codes=True) for _ in range(nl)]
    N, K = synthetic.SHAPES[model]["lm_head"]
    vid, _ = variant_for(lib, kind, N, K, tuned)
    head = Gemv(lib, kind, N, K, g, "lm_head", variant=vid, random_codes=True)
    hy = torch.empty(N, device="cuda", dtype=torch.bfloat16)
    hx = layers[-1].ys[-1][:K]
    plan = None
    if mode == "per_op":
        hcall = head.launcher(hx, hy)

        def token():
            for lay in layers:
                lay.step()
            hcall()
    elif mode == "layer":
        hcall = head.launcher(hx, hy)
        calls = [lay.layer_launcher() for lay in layers]

        def token():
            for c in calls:
                rc = c()
                if rc:
                    raise RuntimeError(f"layer launch failed with code {rc}")
            hcall()
    else:
        ops = [d for lay in layers for d in lay.op_dicts()] + [head.op_dict(hx, hy)]
        plan = lib.plan_create(kind, ops)

        def token():
            lib.plan_launch(plan)
    gph = capture(token)
    for _ in range(3):
        gph.replay()
    torch.cuda.synchronize()
    err = lib.device_error(True)
    if err:
        raise RuntimeError(f"device error {err} in decode_token {kind} {model} {mode}")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    tb = sum(l.weight_bytes() for l in layers) + head.weight_bytes()
    del gph
    if plan is not None:
        lib.plan_destroy(plan)
    out = {"kind": kind, "model": model, "mode": mode, "decode_us_per_token": round(us, 2), "layers": nl,
           "weight_GB": round(tb / 1e9, 3), "GBps": round(tb / us / 1e3, 1),
           "frac_of_peak": round(tb / us / 1e3 / peak, 4)}
    del layers, head
    torch.cuda.empty_cache()
    return out


def run_copy_sweep(args):
    """Copy size against copy count: the TMA kernel on the gate_up shape at explicit ring depths (paia_gemv_launch_ex
    ring option). The stage slot is sized for the ring, so deeper rings mean smaller bulk copies at about the same
    bytes in flight per SM; graph mode over L2-rotated copies."""
    import ctypes
    import torch
    from paia_gemv import load_lib, timing
    torch.cuda.set_device(0)
    lib = load_lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    l2 = timing.l2_bytes()
    P = ctypes.c_void_p
    cur = torch._C._cuda_getCurrentRawStream
    f = lib._lib.paia_gemv_launch_ex
    kid = {"bf16": 0, "fp8": 1, "int4": 2, "int4_asym": 3}
    math_of = {"bf16": 5, "fp8": 8, "int4": 7, "int4_asym": 7}
    N, K = 28672, 4096
    for kind in args.kinds.split(","):
        first = Gemv(lib, kind, N, K, g, "gate_up", variant=0, random_codes=True)
        n = timing.plan_rotation(first.weight_bytes(), l2)
        gms = [first] + [Gemv(lib, kind, N, K, g, "gate_up", variant=0, random_codes=True) for _ in range(n - 1)]
        xs = [torch.randn(K, device="cuda", generator=g).to(torch.bfloat16) for _ in gms]
        ys = [torch.empty(N, device="cuda", dtype=torch.bfloat16) for _ in gms]
        for ring in (0, 3, 4, 6, 8, 12, 16):
            def mk(gm, x, y, ring=ring):
                a = (kid[kind], ring, 2, 8, math_of[kind], 1, 0, 0, P(gm.W.data_ptr()),
                     P(gm.s.data_ptr() if gm.s is not None else 0), P(gm.z.data_ptr() if gm.z is not None else 0),
                     P(x.data_ptr()), None, P(y.data_ptr()), N, K)
                return lambda: f(*a, P(cur(torch.cuda.current_device())))
            calls = [mk(gm, x, y) for gm, x, y in zip(gms, xs, ys)]
            rc = calls[0]()
            torch.cuda.synchronize()
            if rc:
                print(json.dumps({"kind": kind, "ring": ring, "rc": rc}), flush=True)
                continue
            us = timing.median(timing.time_graph(calls, samples=9))
            print(json.dumps({"kind": kind, "N": N, "K": K, "ring": ring, "us": round(us, 2),
                              "GBps": round(first.weight_bytes() / us / 1e3, 1)}), flush=True)
        del gms, xs, ys, first
        torch.cuda.empty_cache()
    return 0


def run_tile_sweep(args):
    """Where a launch's time goes: the default kernel at K = 4096 and 14336 with 1, 2, 4 and 8 tiles (16 rows) per
    CTA (N = 148 x 16 x tiles), cold (weights rotated through more than L2) and hot (one weight copy replayed, when it
    fits in L2), next to the HBM time of its bytes at the measured copy peak. The slope over tiles is the streaming
    cost per tile, the intercept the fixed cost of a launch; hot = cold means the consumers, not HBM, set the pace."""
    import torch
    from paia_gemv import load_lib, timing
    torch.cuda.set_device(0)
    lib = load_lib()
    peak, _ = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(7)
    l2 = timing.l2_bytes()
    for kind in args.kinds.split(","):
        for K in (4096, 14336):
            row = {"kind": kind, "K": K, "cols": ["cold_us", "hot_us", "hbm_us"]}
            for tiles in (1, 2, 4, 8):
                N = 148 * 16 * tiles
                vid, _ = variant_for(lib, kind, N, K, None)
                first = Gemv(lib, kind, N, K, g, "tiles", variant=vid)
                n = max(2, timing.plan_rotation(first.weight_bytes(), l2))
                copies = [first] + [Gemv(lib, kind, N, K, g, "tiles", variant=vid, random_codes=True)
                                    for _ in range(n - 1)]
                xs = [torch.randn(K, device="cuda", generator=g).to(torch.bfloat16) for _ in copies]
                ys = [torch.empty(N, device="cuda", dtype=torch.bfloat16) for _ in copies]
                calls = [c.launcher(x, y) for c, x, y in zip(copies, xs, ys)]
                cold = timing.median(timing.time_graph(calls, samples=9))
                hot = (timing.median(timing.time_graph([calls[0]] * n, samples=9))
                       if first.weight_bytes() < 0.5 * l2 else None)
                row[f"tiles_{tiles}"] = [round(cold, 2), None if hot is None else round(hot, 2),
                                         round(first.weight_bytes() / peak / 1e3, 2)]
                del copies, xs, ys, calls, first
                torch.cuda.empty_cache()
            print(json.dumps(row), flush=True)
    return 0


def run_batched(args):
    """M > 1 activation rows (paia_gemv_batched) on the Llama-3.1-8B shapes: us per call and weight GB/s for M = 1, 2,
    4, 8, 16, graph mode over L2-rotated weight copies, against M separate batch-1 calls of the default path."""
    import ctypes
    import torch
    from paia_gemv import load_lib, synthetic, timing
    from paia_gemv.loader import _KINDS
    torch.cuda.set_device(0)
    lib = load_lib()
    peak, _ = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(7)
    l2 = timing.l2_bytes()
    P = ctypes.c_void_p
    cur = torch._C._cuda_getCurrentRawStream
    fb = lib._lib.paia_gemv_batched
    for kind in args.kinds.split(","):
        for name in ("qkv_fused", "o_proj", "gate_up_fused", "down_proj"):
            N, K = synthetic.SHAPES["llama31_8b"][name]
            vid, _ = variant_for(lib, kind, N, K, None)
            first = Gemv(lib, kind, N, K, g, name, variant=vid, random_codes=True)
            n = timing.plan_rotation(first.weight_bytes(), l2)
            gms = [first] + [Gemv(lib, kind, N, K, g, name, variant=vid, random_codes=True) for _ in range(n - 1)]
            wb = first.weight_bytes()
            for M in (1, 2, 4, 8, 16):
                X = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
                Y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

                def mk(gm):
                    a = (_KINDS[kind], P(gm.W.data_ptr()), P(gm.s.data_ptr() if gm.s is not None else 0),
                         P(gm.z.data_ptr() if gm.z is not None else 0), P(X.data_ptr()), None, P(Y.data_ptr()),
                         M, N, K)
                    return lambda: fb(*a, P(cur(torch.cuda.current_device())))
                calls = [mk(gm) for gm in gms]
                rc = calls[0]()
                torch.cuda.synchronize()
                if rc:
                    print(json.dumps({"kind": kind, "layer": name, "M": M, "rc": rc}), flush=True)
                    continue
                us = timing.median(timing.time_graph(calls, samples=9))
                singles = []
                for gm in gms:
                    for m in range(M):
                        singles.append(gm.launcher(X[m], Y[m]))
                us1 = timing.median(timing.time_graph(singles, samples=9)) * M   # M batch-1 calls
                print(json.dumps({"kind": kind, "model": "llama31_8b", "layer": name, "N": N, "K": K, "M": M,
                                  "us": round(us, 2), "GBps": round(wb / us / 1e3, 1),
                                  "frac_of_peak": round(wb / us / 1e3 / peak, 4),
                                  "us_M_single_calls": round(us1, 2), "speedup": round(us1 / us, 2)}), flush=True)
                del X, Y, calls, singles
            del gms, first
            torch.cuda.empty_cache()
    return 0


def run_decode(args):
    """Decode µs/token of both models in each format, per-op launches vs one launch per layer vs one plan per token."""
    import torch
    from paia_gemv import load_lib
    torch.cuda.set_device(0)
    lib = load_lib()
    tuned = load_tuned()
    peak, _ = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(7)
    for kind in args.kinds.split(","):
        for model in ("llama31_8b", "qwen25_7b"):
            for mode in ("per_op", "layer", "plan"):
                print(json.dumps(decode_token(lib, kind, model, g, tuned, peak, mode)), flush=True)
    return 0


def run_families(args):
    """Per real shape and format: GB/s of each kernel family (TMA-fed tensor-core, register-fed tensor-core,
    CUDA-core instance of the default tuple) through paia_gemv_launch_ex, graph mode over L2-rotated copies. The table
    behind the default path's per-shape choice."""
    import ctypes
    import itertools
    import torch
    from paia_gemv import load_lib, synthetic, timing
    lib = load_lib()
    f = lib._lib.paia_gemv_launch_ex
    P = ctypes.c_void_p
    f.argtypes = [ctypes.c_int] * 8 + [P] * 6 + [ctypes.c_int, ctypes.c_int, P]
    f.restype = ctypes.c_int
    kid = {"bf16": 0, "fp8": 1, "int4": 2, "int4_asym": 3}
    dflt = {"bf16": (2, 4, 4), "fp8": (2, 2, 4), "int4": (4, 2, 4), "int4_asym": (4, 2, 4)}
    tma_math = {"bf16": 5, "fp8": 8, "int4": 7, "int4_asym": 7}
    shapes = sorted({s for m in synthetic.SHAPES.values() for s in m.values()})
    g = torch.Generator(device="cuda").manual_seed(0)
    l2 = timing.l2_bytes()
    for kind in args.kinds.split(","):
        for (N, K) in shapes:
            first = Gemv(lib, kind, N, K, g, "cmp", random_codes=True)
            n = timing.plan_rotation(first.weight_bytes(), l2)
            copies = [first] + [Gemv(lib, kind, N, K, g, "cmp", random_codes=True) for _ in range(n - 1)]
            xs = [torch.randn(K, device="cuda", generator=g).to(torch.bfloat16) for _ in range(n)]
            ys = [torch.empty(N, device="cuda", dtype=torch.bfloat16) for _ in range(n)]
            R, U, W = dflt[kind]
            cfgs = [("tma", 0, 2, 8, tma_math[kind])] + ([("tma_m5", 0, 2, 8, 5)] if kind.startswith("int4") else [])
            cfgs += [(f"mma2_U{u}W{w}", 1, u, w, 2) for u, w in itertools.product((2, 4), (8, 16))]
            cfgs += [("core_m0", R, U, W, 0), ("core_m1", R, U, W, 1)]
            for name, r_, u_, w_, m in cfgs:
                def mk(i, r_=r_, u_=u_, w_=w_, m=m):
                    c = copies[i]
                    a = (kid[kind], r_, u_, w_, m, 1, 0, 0, P(c.W.data_ptr()),
                         P(c.s.data_ptr() if c.s is not None else 0), P(c.z.data_ptr() if c.z is not None else 0),
                         P(xs[i].data_ptr()), None, P(ys[i].data_ptr()), N, K)
                    return lambda: f(*a, P(torch.cuda.current_stream().cuda_stream))
                calls = [mk(i) for i in range(n)]
                rc = calls[0]()
                torch.cuda.synchronize()
                rec = {"kind": kind, "N": N, "K": K, "cfg": name}
                if rc:
                    rec["rc"] = rc
                else:
                    us = timing.median(timing.time_graph(calls, samples=7, target_ms=1.0))
                    rec.update(us=round(us, 3), GBps=round(first.weight_bytes() / us / 1e3, 1))
                print(json.dumps(rec), flush=True)
            del copies, xs, ys, first
            torch.cuda.empty_cache()
    return 0


def run_tp(args, rank, world, local_rank):
    """Row-sharded TP GEMV over the ranks of this launch (torchrun, one process per GPU). For
    Llama-3.1-8B lm_head 128256x4096 and gate_up 28672x4096 in FP8 W8A16 and INT4 (asymmetric) g128: per-call device
    time of the fused path (peer-store epilogue + bounded arrival wait) and of the NCCL all-gather baseline, CUDA
    events around a CUDA graph (fused) or an eager loop (NCCL) over L2-rotated weight shards, max over ranks. One
    JSON line per shape, format and path; GB/s = full weight bytes / time."""
    import datetime
    import torch
    import torch.distributed as dist
    from paia_gemv import load_lib, synthetic, timing, tp
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    else:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29541")
        dist.init_process_group("gloo", rank=0, world_size=1)
    lib = load_lib()
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    l2 = timing.l2_bytes()
    out = []
    for kind in ("fp8", "int4_asym"):
        for name in ("lm_head", "gate_up_fused"):
            N, K = synthetic.SHAPES["llama31_8b"][name]
            r0, r1 = tp.shard_rows(N, world, rank)
            nl = r1 - r0
            first = Gemv(lib, kind, nl, K, g, name, random_codes=True)
            n = timing.plan_rotation(first.weight_bytes(), l2)
            shards = [first] + [Gemv(lib, kind, nl, K, g, name, random_codes=True) for _ in range(n - 1)]
            bufs = tp.TpBuffers(lib, N, torch.device("cuda", local_rank))
            sg = [tp.ShardedGemv(lib, kind, c.W, c.s, c.z, None, N, K, buffers=bufs) for c in shards]
            gx = torch.Generator(device="cuda").manual_seed(7)                 # x is replicated
            x = torch.randn(K, device="cuda", generator=gx).to(torch.bfloat16)
            full_bytes = first.weight_bytes() * world
            reps = max(n, 64 // n * n)

            def fused_round():
                for c in sg:
                    c.fused(x)
            # correctness on this rank: fused y == NCCL y, bit for bit, for the first shard
            yf = sg[0].fused(x).clone()
            yn = sg[0].nccl(x).clone()
            torch.cuda.synchronize()
            same = bool(torch.equal(yf.view(torch.int16), yn.view(torch.int16)))
            graph = capture(fused_round)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps // n):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us_fused = e0.elapsed_time(e1) * 1e3 / (reps // n * n)
            dist.barrier()
            for i in range(2 * n):
                sg[i % n].nccl(x)
            torch.cuda.synchronize()
            dist.barrier()
            e0.record()
            for i in range(reps):
                sg[i % n].nccl(x)
            e1.record()
            torch.cuda.synchronize()
            us_nccl = e0.elapsed_time(e1) * 1e3 / reps
            t = torch.tensor([us_fused, us_nccl, 0.0 if same else 1.0], device="cuda")
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            err = lib.device_error(1)
            del graph
            bufs.close()
            if rank == 0:
                for path, us in (("fused_peer_store", t[0].item()), ("nccl_all_gather", t[1].item())):
                    out.append({"config": "tp_row_sharded", "kind": kind, "layer": name, "N": N, "K": K,
                                "n_gpus": world, "rows_per_rank": nl, "path": path, "us": round(us, 3),
                                "GBps": round(full_bytes / us / 1e3, 1), "fused_equals_nccl": t[2].item() == 0.0,
                                "device_error": err, "timing": "max over ranks, CUDA events, rotated shards"})
                    print(json.dumps(out[-1]), flush=True)
            del sg, shards, first
            torch.cuda.empty_cache()
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_decode_loop(args):
    """Tokens per second of the minimal decode step (paia_gemv.decode): Llama-3.1-8B and Qwen2.5-7B with synthetic
    weights in every format, a 1024-position KV cache, the whole token (GEMVs, norms, RoPE, attention, SiLU x up,
    residuals, lm_head, argmax) as one CUDA graph; next to it the GEMVs alone (decode_token, the same weights bytes)."""
    import torch
    from paia_gemv import decode, load_lib
    torch.cuda.set_device(0)
    lib = load_lib()
    peak, _ = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(7)
    for model in ("llama31_8b", "qwen25_7b"):
        for kind in args.kinds.split(","):
            m = decode.DecodeModel(lib, model, kind, ctx=1024)
            us, ids = decode.time_tokens(m, tokens=20)
            wb = m.weight_bytes()
            del m
            torch.cuda.empty_cache()
            gemv_only = decode_token(lib, kind, model, g, load_tuned(), peak, "per_op", reps=5)
            print(json.dumps({"model": model, "kind": kind, "us_per_token": round(us, 1),
                              "tokens_per_s": round(1e6 / us, 1), "weight_GB": round(wb / 1e9, 3),
                              "GBps_weights": round(wb / us / 1e3, 1),
                              "gemv_only_us_per_token": gemv_only["decode_us_per_token"], "ctx": 1024,
                              "last_token": ids[-1]}), flush=True)
    return 0


# The layer GEMVs of a decode step run back to back, and a chain whose launches switch kernel instances starts each
# launch on code that is not in the instruction cache: measured on B200, the Llama INT4 asym per-op token took 1685 us
# with the per-shape best instances (U = 4 for qkv / gate_up, U = 2 for o / down) and 1386 us with one instance for
# every op (Qwen 1521 -> 1404, INT4 1351 -> 1270 and 1313 -> 1294), while that instance is within 0.2-3.3 % of the
# per-shape best in isolation. So for the integer INT4 formats the GEMVs of a model's decode chain all take the one
# TMA-fed variant that is fastest summed over them. FP8 and BF16 need no rule: their per-shape picks already map to
# one kernel instance.
CHAIN_KINDS = ("int4", "int4_asym")


def chain_rule(tuned, keys, models, chain=None):
    """Apply the decode-chain rule in place: per integer INT4 format and model, the shapes of the decode chain (the
    layer sequence qkv, o, gate_up, down and the lm_head) all take the TMA variant (R = 0) with the lowest summed
    estimated time over them (a shape whose top 5 lacks it counted at its fifth entry's time, a lower bound), ties
    broken by how many top-5 lists hold it. The per-shape pick stays as "isolated_best". Returns
    {(kind, model): variant}."""
    from paia_gemv import synthetic
    chain = chain or synthetic.LAYER_SEQUENCE + ("lm_head",)
    tup = lambda v: tuple(v[k] for k in "RUWSH")                # noqa: E731
    chosen = {}
    for kind in CHAIN_KINDS:
        table = tuned.get(keys[kind], {})
        for model, shapes in models.items():
            entries = [table.get("{}x{}".format(*shapes[name])) for name in chain if name in shapes]
            entries = [e for e in entries if e and e.get("top5")]
            if not entries:
                continue
            cands = {tup(t["variant"]) for e in entries for t in e["top5"] if t["variant"]["R"] == 0}
            scored = []
            for c in sorted(cands):
                hits, total = 0, 0.0
                for e in entries:
                    best_us = e.get("isolated_best", {}).get("us", e["us"])
                    top = e["top5"]
                    pct = next((t["pct_of_best"] for t in top if tup(t["variant"]) == c), None)
                    hits += pct is not None
                    total += best_us * 100.0 / (pct if pct else top[-1]["pct_of_best"])
                scored.append((total, -hits, c))
            if not scored:
                continue
            _, _, c = min(scored)
            var = dict(zip("RUWSH", c))
            for e in entries:
                if "isolated_best" not in e:
                    e["isolated_best"] = {"variant": e["variant"], "us": e["us"]}
                e["variant"] = dict(var)
                e["chain"] = ("one kernel instance for every GEMV of the model's decode chain (decode-chain rule); us, "
                              "gbps and top5 are the isolated per-shape measurements")
            chosen[(kind, model)] = var
    return chosen


def run_tune(args):
    """Per-shape variant choice for B200 written to paia-project_b200/tuned/b200.json in the reference's tuned-table
    schema (src/tools/dev_sweep_bf16.py:90-99: per N x K the best (R, U, W, S, H) with its us and GB/s and the top 5 with
    their % of the best; keys shapes / fp8_shapes / int4_shapes, plus int4_asym_shapes), which bench.py and the
    reference's op adapters (paia-bench ours_bf16.py:32-38, ours_quant.py:29-36, platform tag "b200") read. Every real
    Llama-3.1-8B / Qwen2.5-7B decode shape; graph mode over L2-rotated copies. Candidates: the default tuple, the TMA-fed
    variants (R = 0) and, for N <= 1024 (where the CUDA-core instances run) or with --tune-all, every tuple. A variant
    is kept only if its output matches the default variant's (rel L2 <= 1e-3)."""
    import torch
    from paia_gemv import load_lib, synthetic, timing
    torch.cuda.set_device(0)
    lib = load_lib()
    peak, _ = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(11)
    l2 = timing.l2_bytes()
    out_f = ROOT / "paia-project_b200" / "tuned" / "b200.json"
    tuned = json.loads(out_f.read_text()) if out_f.exists() else {}
    tuned["platform"] = "b200"
    tuned["device"] = torch.cuda.get_device_name(0)
    defaults = {"bf16": (2, 4, 4, 0, 1), "fp8": (2, 2, 4, 0, 1), "int4": (4, 2, 4, 0, 1), "int4_asym": (4, 2, 4, 0, 1)}
    keys = {"bf16": "shapes", "fp8": "fp8_shapes", "int4": "int4_shapes", "int4_asym": "int4_asym_shapes"}
    tables = {"bf16": lib.variants, "fp8": lib.variants_fp8, "int4": lib.variants_int4,
              "int4_asym": lib.variants_int4_asym}
    shapes = sorted({s for m in synthetic.SHAPES.values() for s in m.values()})
    for kind in args.kinds.split(","):
        kmult = {"bf16": 8, "fp8": 16}.get(kind, 128)
        tuned.setdefault(keys[kind], {})
        table = tables[kind]
        tup = lambda v: tuple(v[k] for k in "RUWSH")            # noqa: E731
        dflt = next(v["id"] for v in table if tup(v) == defaults[kind])
        for (N, K) in shapes:
            if K % kmult:
                continue
            cand = [v for v in table if args.tune_all or N <= 1024 or v["R"] == 0 or v["id"] == dflt]
            first = Gemv(lib, kind, N, K, g, "tune", variant=dflt)
            n = timing.plan_rotation(first.weight_bytes(), l2)
            copies = [first] + [Gemv(lib, kind, N, K, g, "tune", variant=dflt, random_codes=True) for _ in range(n - 1)]
            xs = [torch.randn(K, device="cuda", generator=g).to(torch.bfloat16) for _ in copies]
            ys = [torch.empty(N, device="cuda", dtype=torch.bfloat16) for _ in copies]
            first.variant = dflt
            first.launcher(xs[0], ys[0])()
            torch.cuda.synchronize()
            ref = ys[0].float().clone()
            rows = []
            for v in cand:
                for c in copies:
                    c.variant = v["id"]
                calls = [c.launcher(xx, yy) for c, xx, yy in zip(copies, xs, ys)]
                rc = calls[0]()
                torch.cuda.synchronize()
                if rc:
                    continue                                    # the variant cannot run this shape (-2)
                err = ((ys[0].float() - ref).norm() / ref.norm()).item()
                if not err <= 1e-3:
                    print(json.dumps({"kind": kind, "N": N, "K": K, "variant": tup(v), "rejected_rel_l2": err}))
                    continue
                us = timing.median(timing.time_graph(calls, samples=5, target_ms=1.0))
                rows.append((us, v))
            rows.sort(key=lambda r: r[0])
            wb = first.weight_bytes()
            best_us, best = rows[0]
            tuned[keys[kind]][f"{N}x{K}"] = {
                "variant": {k: best[k] for k in "RUWSH"}, "us": round(best_us, 3),
                "gbps": round(wb / best_us / 1e3, 1), "frac_of_peak": round(wb / best_us / 1e3 / peak, 4),
                "top5": [{"variant": {k: v[k] for k in "RUWSH"}, "pct_of_best": round(100 * best_us / us, 1)}
                         for us, v in rows[:5]],
                "candidates": len(rows), "dev_only": True, "when": time.strftime("%Y-%m-%d %H:%M")}
            print(json.dumps({"kind": kind, "N": N, "K": K, "best": tup(best), "us": round(best_us, 3),
                              "default_us": round(next(u for u, v in rows if v["id"] == dflt), 3)}), flush=True)
            del copies, xs, ys, first
            torch.cuda.empty_cache()
    for (kind, model), var in chain_rule(tuned, keys, synthetic.SHAPES).items():
        print(json.dumps({"chain_rule": kind, "model": model, "variant": var}))
    out_f.parent.mkdir(parents=True, exist_ok=True)
    out_f.write_text(json.dumps(tuned, indent=1) + "\n")
    print(json.dumps({"wrote": str(out_f.relative_to(ROOT))}))
    return 0


def run_one(args):
    """A few launches of one shape through the default path (the C ABI call a user makes), for profilers: no timing."""
    import torch
    from paia_gemv import load_lib
    lib = load_lib()
    kind, shape = args.one.split(":")
    N, K = (int(v) for v in shape.split("x"))
    g = torch.Generator(device="cuda").manual_seed(7)
    vid, _ = variant_for(lib, kind, N, K, load_tuned() if args.one_tuned else None)
    gms = [Gemv(lib, kind, N, K, g, "one", variant=vid, random_codes=True) for _ in range(2)]
    x = torch.randn(K, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(N, device="cuda", dtype=torch.bfloat16)
    calls = [gm.launcher(x, y) for gm in gms]
    for i in range(args.launches):
        rc = calls[i % 2]()
        if rc:
            raise RuntimeError(f"launch failed with code {rc}")
    torch.cuda.synchronize()
    print(json.dumps({"one": args.one, "launches": args.launches, "weight_bytes": gms[0].weight_bytes()}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--sweep", action="store_true")
    ap.add_argument("--kinds", default="bf16,fp8,int4,int4_asym")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the 1-GPU extra keys (decode layer, shapes, tokens)")
    ap.add_argument("--one", default=None, help="profiling aid: KIND:NxK, e.g. fp8:28672x4096 (default variant)")
    ap.add_argument("--one-tuned", action="store_true", help="--one with the tuned table's variant (as the bench)")
    ap.add_argument("--families", action="store_true", help="per-shape comparison of the kernel families")
    ap.add_argument("--tp", action="store_true", help="row-sharded TP GEMV over the launched ranks")
    ap.add_argument("--launches", type=int, default=4)
    ap.add_argument("--tune", action="store_true", help="per-shape variant sweep -> paia-project_b200/tuned/b200.json")
    ap.add_argument("--decode-loop", action="store_true",
                    help="tokens/s of the minimal decode step (GEMVs + norms, RoPE, attention, sampling)")
    ap.add_argument("--tune-all", action="store_true", help="with --tune: every tuple on every shape")
    ap.add_argument("--batched", action="store_true", help="M > 1 activation rows (paia_gemv_batched)")
    ap.add_argument("--copy-sweep", action="store_true",
                    help="TMA kernel on gate_up at explicit ring depths (copy size vs copy count)")
    ap.add_argument("--tile-sweep", action="store_true",
                    help="launch time against tiles per CTA, cold and hot (fixed cost vs streaming cost)")
    ap.add_argument("--decode", action="store_true",
                    help="decode us/token: per-op launches vs one launch per layer vs one plan per token")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if args.sweep:
        return run_sweep(args)
    if args.tune:
        return run_tune(args)
    if args.decode_loop:
        return run_decode_loop(args)
    if args.one:
        return run_one(args)
    if args.families:
        return run_families(args)
    if args.decode:
        return run_decode(args)
    if args.tile_sweep:
        return run_tile_sweep(args)
    if args.copy_sweep:
        return run_copy_sweep(args)
    if args.batched:
        return run_batched(args)
    if args.tp:
        return run_tp(args, rank, world, local_rank)
    return run_main(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
