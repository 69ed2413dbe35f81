"""The reference's CPU implementation of the decode GEMV, restated (TEST / BASELINE INFRASTRUCTURE ONLY).

Bejaine/PAIA-Project has no separate CPU GEMV: its CPU-capable path is the torch reference its harness uses to check
every op before timing it (paia-bench/bench/ops/ours_quant.py:69-71, ours_bf16.py:86-87): dequantise W to fp32
(src/paia_gemv/quant.py:16-17, :34-38; the asymmetric INT4 dequantiser of paia-bench/bench/ops/lib_quant.py:226-231),
then y = x.float() @ Wdeq[r:r+REF_ROWS].t() in chunks of REF_ROWS = 8192 rows (paia-bench/bench/ops/cublas_bf16.py:11),
with torch's CPU kernels on all host threads. The op dequantises once when it is built (ours_quant.py:99, :138) and
each check runs only the chunked matmul, so the timed per-call work is `matmul` and the dequantisation is reported
apart. This module reproduces that path step for step so that bench.py can
time it on the GPU box's own host cores (where the reference checkout does not exist) as the CPU baseline and as the
`--impl reference` arm. It is never the product: the product path is the CUDA library.
"""
import os
import time

import torch

REF_ROWS = 8192


def set_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def dequant(kind, W, s=None, z=None):
    """fp32 dequantised rows, exactly as the reference's quant.py / lib_quant.py compute them."""
    if kind == "bf16":
        return W.float()
    if kind == "fp8":
        return W.view(torch.float8_e4m3fn).float() * s[:, None]
    p = W.to(torch.int32)
    n = torch.stack([p & 0xF, p >> 4], dim=-1).view(W.shape[0], W.shape[1] * 2).float()
    if kind == "int4":
        return (n - 8.0) * s.float().repeat_interleave(128, dim=1)
    return (n - 8.0) * s.float().repeat_interleave(128, dim=1) + z.float().repeat_interleave(128, dim=1)


def matmul(x, deq):
    """y = x.float() @ deq^T in chunks of REF_ROWS rows: the reference's per-call CPU work (ours_quant.py:69-71), which
    runs on weights dequantised once when the op is built (ours_quant.py:99, :138)."""
    xf = x.float()[None, :]
    return torch.cat([xf @ deq[r:r + REF_ROWS].t() for r in range(0, deq.shape[0], REF_ROWS)], dim=1)[0]


def gemv(kind, x, W, s=None, z=None):
    """(y fp32 [N], seconds in dequantisation, seconds in the matmul) of one dequantise-then-matmul."""
    t0 = time.perf_counter()
    deq = dequant(kind, W, s, z)
    t1 = time.perf_counter()
    y = matmul(x, deq)
    t2 = time.perf_counter()
    return y, t1 - t0, t2 - t1


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"
