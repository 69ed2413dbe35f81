#!/usr/bin/env python
"""Benchmark of the B200 batch-1 decode GEMV family (the driver's contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}] [--sweep]

Workload (the one the headline metric is quoted on): the Llama-3.1-8B FP8 W8A16 decode-layer GEMV
sequence at batch 1 -- qkv 6144x4096 -> o 4096x4096 -> gate_up 28672x4096 -> down 4096x14336, each GEMV reading the
previous one's output as x (o reads qkv[:4096], down reads gate_up[:14336]). One step = one decode layer (4 launches).
Weights ~ N(0, 0.02) quantised to e4m3 with a per-row fp32 scale, x ~ N(0, 1) bf16, synthetic (no checkpoints).
The steps rotate over L distinct layers (L * 208 MiB > 4 x L2), so weights always stream from HBM.

value   = algorithmic bytes (e4m3 weights + fp32 row scales) of all steps / device time of the K steps, GB/s,
          max over ranks; at N > 1 every rank runs its own layers (weak scaling, no data-path collective).
e2e     = the same metric through the public Python API (ctypes -> C ABI, eager launches), with each step's x copied
          host->device from pinned memory and the layer output copied device->host inside the timed region; the
          copies overlap the neighbouring steps' compute on two copy streams (serial_value: all on one stream).
roofline: the dominant (and only) kernel of the step is the FP8 GEMV kernel; achieved = algorithmic bytes / time.
cpu_baseline: the reference's CPU path (dequantise + chunked fp32 matmul, oracle/cpu_reference.py) on the host cores.
--impl reference: that CPU path alone, as the reference arm (rank 0 only).
--sweep: per-shape / per-format / per-model table as JSON lines, plus decode us/token.
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

METRIC = "GEMV achieved HBM GB/s, Llama-3.1-8B FP8 W8A16 decode-layer sweep (qkv, o, gate_up, down), batch 1"
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


# ----------------------------------------------------------------------------------------------- CPU baseline

def cpu_layer_operands(kind="fp8", model="llama31_8b", seed=0):
    """Seeded CPU operands of one decode layer: (name, N, K, W, s, z, x) per GEMV."""
    import torch
    from paia_gemv import quant, synthetic
    g = synthetic.generator(seed)
    ops = []
    for name in synthetic.LAYER_SEQUENCE:
        N, K = synthetic.SHAPES[model][name]
        W = synthetic.weights_f32(N, K, g)
        x = synthetic.activation_bf16(K, g)
        if kind == "fp8":
            q, s = quant.quantize_fp8_rowwise(W)
            ops.append((name, N, K, q, s, None, x))
        elif kind == "bf16":
            ops.append((name, N, K, W.to(torch.bfloat16), None, None, x))
        elif kind == "int4":
            p, s = quant.quantize_int4_g128(W)
            ops.append((name, N, K, p, s, None, x))
        else:
            p, s, z = quant.quantize_int4_asym(W)
            ops.append((name, N, K, p, s, z, x))
        del W
    return ops


def cpu_run_layer(ops, frac, kind="fp8"):
    """The reference's CPU path over the first frac of every GEMV's rows; returns (bytes, dequant s, matmul s)."""
    import cpu_reference as C
    nbytes, td, tm = 0, 0.0, 0.0
    for (name, N, K, W, s, z, x) in ops:
        rows = max(1, int(round(N * frac)))
        Wr = W[:rows]
        sr = None if s is None else s[:rows]
        zr = None if z is None else z[:rows]
        _, a, b = C.gemv(kind, x, Wr, sr, zr)
        td += a
        tm += b
        nbytes += Wr.numel() * Wr.element_size() + sum(t.numel() * t.element_size() for t in (sr, zr) if t is not None)
    return nbytes, td, tm


def cpu_baseline(target_s=15.0, kind="fp8"):
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_reference as C
    threads = C.set_threads()
    ops = cpu_layer_operands(kind)
    t0 = time.perf_counter()
    cpu_run_layer(ops, 1.0, kind)               # warm-up and calibration
    t_layer = time.perf_counter() - t0
    frac = 1.0 if t_layer * 3 <= target_s else max(0.02, target_s / 3 / t_layer)
    reps = max(3, min(20, int(target_s / max(t_layer * frac, 1e-3))))
    times, tds, tms, nb = [], [], [], 0
    for _ in range(reps):
        t0 = time.perf_counter()
        nb, td, tm = cpu_run_layer(ops, frac, kind)
        times.append(time.perf_counter() - t0)
        tds.append(td)
        tms.append(tm)
    med = statistics.median(times)
    return {"value": nb / med / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": (f"{'all' if frac == 1.0 else f'{frac:.3f} of the'} rows of one Llama-3.1-8B {kind} decode layer "
                       f"(qkv, o, gate_up, down; {nb / 2**20:.1f} MiB): dequantise + fp32 matmul in 8192-row chunks "
                       f"(the reference harness's CPU reference path), median of {reps} reps after 1 warm-up; "
                       f"dequant {statistics.median(tds) * 1e3:.1f} ms + matmul {statistics.median(tms) * 1e3:.1f} ms "
                       f"per rep; CPU {C.cpu_model()}, torch threads {threads}, os.cpu_count {os.cpu_count()}"),
            "ms_per_layer": med * 1e3 / frac}


# ----------------------------------------------------------------------------------------------- arms

def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU implementation on this host's cores; rank 0 only."""
    if rank != 0:
        return 0
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_reference as C
    threads = C.set_threads()
    ops = cpu_layer_operands("fp8")
    t0 = time.perf_counter()
    cpu_run_layer(ops, 1.0)
    t_layer = time.perf_counter() - t0
    budget = 150.0
    frac = min(1.0, budget / max(1, args.steps + args.warmup) / t_layer)
    frac = max(frac, 1e-3)
    for _ in range(args.warmup):
        cpu_run_layer(ops, frac)
    nbytes = 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        nb, _, _ = cpu_run_layer(ops, frac)
        nbytes += nb
    dt = time.perf_counter() - t0
    value = nbytes / dt / 1e9
    sample = (f"each step: {frac:.4f} of the rows of every GEMV of one Llama-3.1-8B FP8 decode layer "
              f"({nbytes / args.steps / 2**20:.2f} MiB), dequantise + fp32 matmul in 8192-row chunks (the reference "
              f"harness's CPU reference path, restated in oracle/cpu_reference.py); CPU {C.cpu_model()}, "
              f"{threads} torch threads")
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantised to e4m3, N(0,1) bf16 x)",
            "config": {"workload": "llama31_8b fp8 w8a16 decode-layer GEMV sweep, batch 1", "device": "cpu"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_main(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from paia_gemv import load_lib, synthetic, timing
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    lib = load_lib()
    tuned = load_tuned()
    kind, model = "fp8", "llama31_8b"
    g = torch.Generator(device="cuda").manual_seed(1000 * rank + 1)
    l2 = timing.l2_bytes()
    probe = Layer(lib, kind, model, g, tuned)
    lbytes = probe.weight_bytes()
    L = max(4, math.ceil(4 * l2 / lbytes))
    layers = [probe] + [Layer(lib, kind, model, g, tuned) for _ in range(L - 1)]
    check_err = check_layer(layers[0])
    if not check_err <= 1e-3:
        raise RuntimeError(f"device sanity check failed: rel L2 {check_err:.3e} against torch fp32")

    def run_steps(n):
        for i in range(n):
            layers[i % L].step()

    # graphs: one full rotation (L steps) and a tail, so exactly K (or W) steps run
    g_round = capture(lambda: run_steps(L))
    tails = {}

    def replay(n):
        for _ in range(n // L):
            g_round.replay()
        r = n % L
        if r:
            if r not in tails:
                tails[r] = capture(lambda: run_steps(r))
            tails[r].replay()

    if args.steps % L:
        tails[args.steps % L] = capture(lambda: run_steps(args.steps % L))
    if args.warmup % L and args.warmup % L not in tails:
        tails[args.warmup % L] = capture(lambda: run_steps(args.warmup % L))
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
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    sampler.stop()
    clocks = sampler.summary(t_host0, t_host1)
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = t.item()
    total_bytes = lbytes * args.steps * world
    value = total_bytes / (ms_max * 1e-3) / 1e9
    launches = 4 * args.steps * world

    # per-shape GEMV microseconds (graph mode, each shape alone, L2-rotated random-code copies)
    per_shape = {}
    for gi, name in enumerate(synthetic.LAYER_SEQUENCE):
        N, K = synthetic.SHAPES[model][name]
        ref = layers[0].gemvs[gi]
        n = timing.plan_rotation(ref.weight_bytes(), l2)
        copies = [ref] + [Gemv(lib, kind, N, K, g, name, variant=ref.variant, random_codes=True) for _ in range(n - 1)]
        xs = [torch.randn(K, device="cuda", generator=g).to(torch.bfloat16) for _ in copies]
        ys = [torch.empty(N, device="cuda", dtype=torch.bfloat16) for _ in copies]
        calls = [c.launcher(x, y) for c, x, y in zip(copies, xs, ys)]
        us = timing.median(timing.time_graph(calls, samples=15))
        wb = ref.weight_bytes()
        per_shape[name] = {"N": N, "K": K, "us": round(us, 3), "GBps": round(wb / us / 1e3, 1),
                           "variant": layers[0].gemvs[gi].variant}
        del copies, xs, ys, calls
    torch.cuda.empty_cache()

    # e2e through the public API with host buffers: eager launches, every step's x copied host->device from pinned
    # memory and its layer output device->host, one sync at the end. Headline: the copies on two copy streams, so a
    # step's input lands while the previous step computes and its output drains while the next one does (events
    # order each copy against the compute that reads or overwrites its buffer). Also reported: all on one stream.
    x_host = torch.empty(layers[0].x.numel(), dtype=torch.bfloat16).pin_memory()
    x_host.copy_(layers[0].x.cpu())
    y_host = torch.empty(layers[0].ys[-1].numel(), dtype=torch.bfloat16).pin_memory()
    main = torch.cuda.current_stream()
    main_h = main.cuda_stream
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    done = [torch.cuda.Event() for _ in range(L)]       # layer slot's step finished (its x read, its output written)
    x_in = [torch.cuda.Event() for _ in range(L)]       # layer slot's x landed
    y_out = [torch.cuda.Event() for _ in range(L)]      # layer slot's output copied out

    def copy_on(stream, dst, src):
        torch.cuda.set_stream(stream)                   # ~5 us of host time; the stream context manager takes ~16
        dst.copy_(src, non_blocking=True)
        torch.cuda.set_stream(main)

    def h2d(i):
        j = i % L
        s_in.wait_event(done[j])                        # step i - L has read this slot's x
        copy_on(s_in, layers[j].x, x_host)
        x_in[j].record(s_in)

    def piped_step(i):
        j = i % L
        lay = layers[j]
        main.wait_event(x_in[j])
        main.wait_event(y_out[j])                       # step i - L's output has been copied out
        lay.step_api(main_h)
        done[j].record(main)
        s_out.wait_event(done[j])
        copy_on(s_out, y_host, lay.ys[-1])
        y_out[j].record(s_out)
        h2d(i + 1)                                      # the next step's input, behind this step's compute

    def serial_step(i):
        lay = layers[i % L]
        lay.x.copy_(x_host, non_blocking=True)
        lay.step_api()
        y_host.copy_(lay.ys[-1], non_blocking=True)

    def e2e_time(step, first):
        for i in range(args.warmup):
            step(first + i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for i in range(args.steps):
            step(first + args.warmup + i)
        a1.record()
        torch.cuda.synchronize()
        t = a0.elapsed_time(a1)
        if world > 1:
            t = torch.tensor([t], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t = t.item()
        return t

    e2e_serial_ms = e2e_time(serial_step, 0)
    h2d(0)
    e2e_ms = e2e_time(piped_step, 0)
    main.wait_stream(s_in)
    main.wait_stream(s_out)
    torch.cuda.synchronize()
    if not bool(torch.isfinite(y_host.float()).all()):
        raise RuntimeError("e2e: non-finite layer output copied to the host")
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    e2e_serial_value = total_bytes / (e2e_serial_ms * 1e-3) / 1e9

    peak, peak_src = measured_peaks()
    # roofline of the dominant kernel (gate_up: over half of the layer's bytes), from its per-launch device time
    dom = per_shape["gate_up_fused"]
    dom_bytes = layers[0].gemvs[synthetic.LAYER_SEQUENCE.index("gate_up_fused")].weight_bytes()
    achieved = dom_bytes / (dom["us"] * 1e-6) / 1e9
    traffic = kernel_traffic()
    result = None
    if rank == 0:
        cb = None
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_baseline()
            cb = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in cb.items() if k != "ms_per_layer"}
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp8 e4m3 weights x bf16 x, fp32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) weights quantised to e4m3 + fp32 row scale, N(0,1) bf16 x)",
            "config": {"workload": "llama31_8b fp8 w8a16 decode-layer GEMV sweep: qkv 6144x4096 -> o 4096x4096 -> "
                                   "gate_up 28672x4096 -> down 4096x14336, batch 1, chained",
                       "layers_rotated": L, "bytes_per_step": lbytes,
                       "l2": f"inputs larger than L2: rotation over {L} layers = {L * lbytes / 2**20:.0f} MiB "
                             f"> 4 x L2 ({l2 / 2**20:.0f} MiB)",
                       "launch": "CUDA graph of back-to-back launches with programmatic dependent launch",
                       "per_gpu_layers": "each rank streams its own layers" if world > 1 else None},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src + " (burst copy)",
                         "traffic": (traffic or {}).get("fp8_gate_up_dram_bytes_per_launch"),
                         "algorithmic_bytes_per_launch": dom_bytes,
                         "kernel": "pb2::gemv_tma_kernel<FP8, 8, 2, 3> (gate_up 28672x4096: e4m3 weights + fp32 "
                                   "row scales per launch, timed per launch with CUDA events over L2-rotated copies)",
                         "layer_achieved": round(lbytes * args.steps / (ms * 1e-3) / 1e9, 1)},
            "per_shape_us": per_shape,
            "us_per_layer": round(ms_max * 1e3 / args.steps, 3),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": layers[0].x.numel() * 2,
                    "d2h_bytes_per_step": layers[0].ys[-1].numel() * 2,
                    "serial_value": round(e2e_serial_value, 2),
                    "how": "public API (paia_gemv.loader ctypes -> C ABI), eager launches; per step pinned H2D of x, "
                           "4 GEMVs, D2H of the layer output; CUDA events around all K steps. value: the copies on "
                           "two copy streams (step i+1's input lands while step i computes, step i's output drains "
                           "while step i+1 computes; events order every copy against the compute that reads or "
                           "overwrites its buffer). serial_value: copies and GEMVs in order on one stream"},
            "gpu_launches": launches,
            "clocks": clocks,
            "check_rel_l2_vs_torch": round(check_err, 6),
        }
        if cb is not None:
            result["cpu_baseline"] = cb
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)
    return 0


def run_sweep(args):
    """All BASELINE configs 1-4 per shape and format (graph mode, L2 rotation), one JSON line each, plus the decode
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
    """row-sharded TP GEMV over the ranks of this launch (torchrun, one process per GPU). For
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


def run_one(args):
    """A few launches of one shape through the default path (the C ABI call a user makes), for profilers: no timing."""
    import torch
    from paia_gemv import load_lib
    lib = load_lib()
    kind, shape = args.one.split(":")
    N, K = (int(v) for v in shape.split("x"))
    g = torch.Generator(device="cuda").manual_seed(7)
    vid, _ = variant_for(lib, kind, N, K, None)
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
    ap.add_argument("--one", default=None, help="profiling aid: KIND:NxK, e.g. fp8:28672x4096 (default variant)")
    ap.add_argument("--families", action="store_true", help="per-shape comparison of the kernel families")
    ap.add_argument("--tp", action="store_true", help="row-sharded TP GEMV over the launched ranks (config 5)")
    ap.add_argument("--launches", type=int, default=4)
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
