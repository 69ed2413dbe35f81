"""Generate the golden vectors in tests/golden/golden_v1.npz from the REFERENCE'S OWN CODE.

Run where the read-only reference checkout exists ($PAIA_REFERENCE, else a directory named "reference" beside this
repository):

    python tests/golden/make_golden.py

It imports, unmodified and on the CPU:
  * src/paia_gemv/quant.py            quantize_fp8_rowwise, dequant_fp8, quantize_int4_g128, dequant_int4 (:8-38)
  * paia-bench/bench/ops/lib_quant.py _quant_int4_asym (:159-167), the only definition of the asymmetric format
  * src/tests/emulate_formats.py      fp8_kernel_math / int4_kernel_math: numpy ports of the reference KERNELS'
                                      fp32 dataflow (:70-99, :136-172), i.e. what the reference GPU kernels compute
and records, for seeded operands (paia_gemv.synthetic, CPU generator):
  * the quantised bytes and scales the reference produces,
  * the reference harness's fp32 torch reference y = x.float() @ dequant(W).t() (ours_quant.py:69-71),
  * the reference kernels' fp32 result (emulated dataflow) for FP8 and INT4,
so that tests can pin the oracle (and the CUDA kernels) to the reference on machines where the reference is absent.
Large operands are not stored: they are regenerated from the seed and checked against a stored SHA-256.
"""
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
REF = Path(os.environ["PAIA_REFERENCE"]) if os.environ.get("PAIA_REFERENCE") else ROOT.parent / "reference"
sys.path.insert(0, str(ROOT / "paia-project_b200"))
sys.path.insert(0, str(REF / "paia-bench"))

from paia_gemv import synthetic  # noqa: E402  (the product's seeded generator)
import importlib.util  # noqa: E402


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


ref_quant = _load("ref_quant", REF / "src" / "paia_gemv" / "quant.py")
from bench.ops import lib_quant  # noqa: E402
emu = _load("emulate_formats", REF / "src" / "tests" / "emulate_formats.py")

OUT = Path(__file__).resolve().parent / "golden_v1.npz"


def bits16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_y(x, Wdeq):
    # ours_quant.py:69-71 / ours_bf16.py:86-87, without the REF_ROWS chunking (rows are independent).
    return (x.float()[None, :] @ Wdeq.float().t())[0].numpy().astype(np.float32)


def main():
    rec = {}
    # (N, K, seed, store_W): BF16 shapes include the reference's awkward ones (test_gemv_bf16.py:16).
    bf16_cases = [(1, 8, 11, True), (1, 256, 12, True), (3, 264, 13, True), (7, 520, 14, True), (33, 1032, 15, True),
                  (129, 4104, 16, False), (64, 4096, 0, False)]
    quant_cases = [(1, 128, 21, True), (5, 384, 22, True), (16, 256, 23, True), (33, 1152, 24, False),
                   (64, 4096, 0, False), (24, 3584, 25, False)]
    names = []
    for (N, K, seed, store) in bf16_cases:
        key = f"bf16_{N}x{K}_s{seed}"
        W, x, b = synthetic.operands(N, K, seed=seed, with_bias=True)
        Wb = W.to(torch.bfloat16)
        rec[f"{key}/x"] = bits16(x)
        rec[f"{key}/bias"] = bits16(b)
        rec[f"{key}/W_sha"] = np.array(sha(bits16(Wb)))
        if store:
            rec[f"{key}/W"] = bits16(Wb)
        rec[f"{key}/y_ref_fp32"] = ref_y(x, Wb)
        names.append(key)
    for (N, K, seed, store) in quant_cases:
        W, x, b = synthetic.operands(N, K, seed=seed, with_bias=True)
        # FP8 (quant.py:8-17)
        key = f"fp8_{N}x{K}_s{seed}"
        q, s = ref_quant.quantize_fp8_rowwise(W)
        rec[f"{key}/x"] = bits16(x); rec[f"{key}/bias"] = bits16(b)
        rec[f"{key}/W_sha"] = np.array(sha(W.numpy()))
        if store:
            rec[f"{key}/W"] = W.numpy()
        rec[f"{key}/q"] = q.numpy(); rec[f"{key}/scale"] = s.numpy()
        rec[f"{key}/y_ref_fp32"] = ref_y(x, ref_quant.dequant_fp8(q, s))
        xb = bits16(x).astype(np.uint32)
        yk, cover = emu.fp8_kernel_math(q.numpy(), s.numpy(), xb, R=2, U=2)
        assert (cover == 1).all()
        rec[f"{key}/y_refkernel_fp32"] = np.asarray(yk, dtype=np.float32)
        names.append(key)
        # INT4 symmetric (quant.py:20-38)
        key = f"int4_{N}x{K}_s{seed}"
        p, s16 = ref_quant.quantize_int4_g128(W)
        rec[f"{key}/x"] = bits16(x); rec[f"{key}/bias"] = bits16(b)
        rec[f"{key}/W_sha"] = np.array(sha(W.numpy()))
        if store:
            rec[f"{key}/W"] = W.numpy()
        rec[f"{key}/packed"] = p.numpy(); rec[f"{key}/scales"] = bits16(s16)
        rec[f"{key}/y_ref_fp32"] = ref_y(x, ref_quant.dequant_int4(p, s16))
        yk, cover = emu.int4_kernel_math(p.numpy(), bits16(s16).view(np.float16), xb, R=2, U=2)
        assert (cover == 1).all()
        rec[f"{key}/y_refkernel_fp32"] = np.asarray(yk, dtype=np.float32)
        names.append(key)
        # INT4 asymmetric (lib_quant.py:159-167; bf16 scale/zero as the kernel reads them, :209 and :227)
        key = f"int4a_{N}x{K}_s{seed}"
        qa, sa, za = lib_quant._quant_int4_asym(W)
        qa = qa.to(torch.int32)
        pa = (qa[:, 0::2] | (qa[:, 1::2] << 4)).to(torch.uint8)      # even k in the LOW nibble (this repo's layout)
        sb, zb = sa.to(torch.bfloat16), za.to(torch.bfloat16)
        rec[f"{key}/x"] = bits16(x); rec[f"{key}/bias"] = bits16(b)
        rec[f"{key}/W_sha"] = np.array(sha(W.numpy()))
        if store:
            rec[f"{key}/W"] = W.numpy()
        rec[f"{key}/packed"] = pa.numpy(); rec[f"{key}/scales"] = bits16(sb); rec[f"{key}/zeros"] = bits16(zb)
        # the dequantiser of TinygemmInt4.check (lib_quant.py:226-231), in fp32
        G = K // 128
        deq = ((qa.view(N, G, 128).float() - 8) * sb.float()[:, :, None] + zb.float()[:, :, None]).view(N, K)
        rec[f"{key}/y_ref_fp32"] = ref_y(x, deq)
        names.append(key)
    # Special values from the reference's GPU test (src/tests/test_gemv_bf16.py:26-29): zero W, large W and x.
    g = torch.Generator().manual_seed(5)
    Ws = ((torch.rand(40, 3584, generator=g) - 0.5) * 0.04).to(torch.bfloat16)
    xs = (torch.rand(3584, generator=g) - 0.5).to(torch.bfloat16)
    Wl = (Ws.float() * 1e4).clamp(-3e4, 3e4).to(torch.bfloat16)
    xl = (xs.float() * 1e2).to(torch.bfloat16)
    for key, Wk, xk in (("special_zeros", torch.zeros_like(Ws), xs), ("special_large", Wl, xl)):
        rec[f"{key}/W"] = bits16(Wk); rec[f"{key}/x"] = bits16(xk)
        rec[f"{key}/y_ref_fp32"] = ref_y(xk, Wk)
        names.append(key)
    rec["cases"] = np.array(names)
    rec["provenance"] = np.array("generated by tests/golden/make_golden.py from the reference's quant.py, lib_quant.py "
                                 f"and emulate_formats.py; torch {torch.__version__}")
    np.savez_compressed(OUT, **rec)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.0f} KiB, {len(names)} cases)")


if __name__ == "__main__":
    main()
