"""Device timing of GEMV calls: the reference harness's graph-mode protocol (paia-bench/bench/timing.py:18-173) in
compact form.

* L2 rotation: n_copies = max(2, ceil(factor * L2 / footprint)) independent operand sets, capped by a memory budget,
  so that consecutive calls read distinct memory and the reuse distance exceeds `factor` x L2 (126 MB on B200).
* graph mode: R back-to-back calls (cycling through the copies) are captured in one CUDA graph; CUDA events around
  each replay give per-call microseconds = elapsed / R. Back-to-back launches in one graph are what a decode step
  issues, and programmatic dependent launch overlaps each GEMV's weight stream with its predecessor's tail.
"""
import math
import statistics

import torch


def l2_bytes(device=None):
    return torch.cuda.get_device_properties(device if device is not None else torch.cuda.current_device()).L2_cache_size


def plan_rotation(footprint, l2=None, factor=4, mem_cap_bytes=48 << 30):
    l2 = l2 or l2_bytes()
    want = max(2, math.ceil(factor * l2 / max(footprint, 1)))
    fit = max(1, mem_cap_bytes // max(footprint, 1))
    return min(want, fit)


def capture(calls, R):
    """CUDA graph of R calls, cycling through `calls` (a list of zero-argument launch functions)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for j in range(min(3, R)):
            calls[j % len(calls)]()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for j in range(R):
            calls[j % len(calls)]()
    return g


def time_graph(calls, R=None, samples=20, warmup=3, target_ms=2.0):
    """Per-call microseconds (list of `samples` values) of `calls` replayed back to back in a CUDA graph."""
    if R is None:
        g = capture(calls, len(calls))
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(); g.replay(); e1.record(); e1.synchronize()
        per = e0.elapsed_time(e1) / len(calls)
        R = max(len(calls), int(math.ceil(target_ms / max(per, 1e-4) / len(calls))) * len(calls))
        R = min(R, 4096)
        del g
    g = capture(calls, R)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(samples)]
    for a, b in ev:
        a.record()
        g.replay()
        b.record()
    torch.cuda.synchronize()
    out = [a.elapsed_time(b) * 1e3 / R for a, b in ev]
    del g
    return out


def median(xs):
    return statistics.median(xs)
