"""Harness integration: time this library's GEMVs with the reference's unchanged cell runner (paia-bench bench.run).

The runner (paia-bench/bench/run.py) looks phases up in its module-level PHASES table and builds ops in
GpuContext.make_op; phases for the quantised GEMVs were added to it by a patch (src/patches/integration_quant.patch)
that no longer applies to the current runner. `register(run)` adds them from outside instead, without editing the
runner:

  s3  FP8 W8A16 (the reference adapter bench.ops.ours_quant.OursFP8Gemv), every timing mode
  s4  INT4 W4A16 g128 fused in every timing mode, plus the naive and unfused controls in graph mode
      (bench.ops.ours_quant.OursInt4Gemv)
  s5  asymmetric INT4 g128 (no reference adapter: `Int4AsymGemv` below, same conventions), every timing mode

over the runner's synthetic sweep and every model shape whose K the format accepts, M = 1. The adapters import
`paia_gemv` (load_lib, quant); with this package first on sys.path that is this library, so the runner times the
B200 kernels through the same C ABI calls a user makes.

    PAIA_BENCH=<paia-bench dir> python -m paia_gemv.harness --phase s3 --session S [runner options]
"""
import os
import sys
from pathlib import Path

_PKG_PARENT = Path(__file__).resolve().parent.parent

MODES = ("isolated", "eager", "graph")


def quant_cells(cfg, phase, impl, precision, kmult, modes):
    """Cells of one quantised-GEMV implementation: the synthetic sweep and every model shape with K % kmult == 0, at
    M = 1 (the shape and field layout the runner's other GEMV phases use)."""
    base = {"phase": phase, "op": "linear", "impl": impl, "precision": precision, "hot_or_cold": "cold"}
    cells = []
    for name, sweep in cfg["synthetic"].items():
        if sweep["K"] % kmult:
            continue
        for n in sweep["N"]:
            for mode in modes:
                cells.append({**base, "shape": {"M": 1, "N": n, "K": sweep["K"]}, "model": "synthetic",
                              "layer_name": f"{name}_N{n}", "timing_mode": mode})
    for model, m in cfg["models"].items():
        for layer, (n, k) in m["shapes"].items():
            if k % kmult:
                continue
            for mode in modes:
                cells.append({**base, "shape": {"M": 1, "N": n, "K": k}, "model": model, "layer_name": layer,
                              "timing_mode": mode})
    return cells


def phases(config):
    """{phase: cell generator} for the runner's PHASES table; `config` is the runner's bench.config module."""
    def s3():
        return quant_cells(config.shapes_cfg(), "s3", "ours_fp8_w8a16", "fp8_w8a16", 16, MODES)

    def s4():
        cfg = config.shapes_cfg()
        return (quant_cells(cfg, "s4", "ours_int4_fused", "int4_g128_w4a16", 128, MODES)
                + quant_cells(cfg, "s4", "ours_int4_naive", "int4_g128_w4a16", 128, ("graph",))
                + quant_cells(cfg, "s4", "ours_int4_unfused", "int4_g128_w4a16", 128, ("graph",)))

    def s5():
        return quant_cells(config.shapes_cfg(), "s5", "ours_int4_asym", "int4_asym_g128_w4a16", 128, MODES)

    return {"s3": s3, "s4": s4, "s5": s5}


def int4_asym_op():
    """The harness Op for the asymmetric INT4 format (bench.ops.base.Op subclass, built on first use because the base
    class lives in the harness). Conventions of the reference's quantised adapters (bench/ops/ours_quant.py): M = 1,
    copy 0 quantised from the shared uniform(-0.02, 0.02) weights with the same seed, its fp32 dequantisation as the
    reference and the harness gate max|y - ref| / max|ref| < 2e-2, copies 1.. valid random codes for L2 rotation,
    bytes() counting weights plus scale and zero metadata."""
    import torch
    from bench.ops.base import Op

    class Int4AsymGemv(Op):
        op, impl, precision = "linear", "ours_int4_asym", "int4_asym_g128_w4a16"

        def __init__(self, M=None, N=None, K=None, model=None, layer_name=None, variant=None, platform_tag=None):
            if M != 1:
                raise NotImplementedError("ours_int4_asym supports M=1 only")
            if K % 128:
                raise ValueError("K % 128 required")
            super().__init__(M, N, K, model, layer_name)
            from paia_gemv import load_lib
            self.lib = load_lib()
            want = {"R": 4, "U": 2, "W": 4, "S": 0, "H": 1}     # the INT4 adapters' default tuple
            self.variant = int(variant) if variant is not None else next(
                v["id"] for v in self.lib.variants_int4_asym if all(v[k] == want[k] for k in "RUWSH"))

        def impl_config(self):
            return {"variant": self.lib.variants_int4_asym[self.variant], "variant_source": "default"}

        def footprint_bytes(self):
            return self.N * self.K // 2 + 4 * self.N * (self.K // 128) + 2 * self.K + 2 * self.N

        def bytes(self):
            return {"weights": self.N * self.K // 2, "metadata": 4 * self.N * (self.K // 128),
                    "act_in": 2 * self.M * self.K, "out": 2 * self.M * self.N}

        def build(self, n_copies):
            from paia_gemv.quant import dequant_int4_asym, quantize_int4_asym
            g = torch.Generator(device="cuda").manual_seed(1000 + self.N + self.K)
            W0 = (torch.rand(self.N, self.K, device="cuda", generator=g, dtype=torch.float32) - 0.5).mul_(0.04)
            self._tx = [(torch.rand(self.M, self.K, device="cuda", generator=g) - 0.5).to(torch.bfloat16)
                        for _ in range(n_copies)]
            self._ty = [torch.empty(self.M, self.N, device="cuda", dtype=torch.bfloat16) for _ in range(n_copies)]
            p0, s0, z0 = quantize_int4_asym(W0)
            self._ref_deq = dequant_int4_asym(p0, s0, z0)
            del W0
            G = self.K // 128
            self._tq = [p0] + [torch.randint(0, 256, (self.N, self.K // 2), device="cuda", dtype=torch.uint8)
                               for _ in range(n_copies - 1)]
            self._ts = [s0] + [(torch.rand(self.N, G, device="cuda") * 1e-3 + 1e-4).to(torch.bfloat16)
                               for _ in range(n_copies - 1)]
            self._tz = [z0] + [(torch.randn(self.N, G, device="cuda") * 1e-3).to(torch.bfloat16)
                               for _ in range(n_copies - 1)]
            self._tptrs = [(q.data_ptr(), s.data_ptr(), z.data_ptr(), x.data_ptr(), y.data_ptr())
                           for q, s, z, x, y in zip(self._tq, self._ts, self._tz, self._tx, self._ty)]

        def call(self, i):
            q, s, z, x, y = self._tptrs[i]
            self.lib.int4_asym(q, s, z, x, y, self.N, self.K, self.variant)
            return self._ty[i]

        def check(self):
            self._ty[0].zero_()
            y = self.call(0).float()
            x = self._tx[0].float()
            ref = torch.cat([x @ self._ref_deq[r:r + 8192].t() for r in range(0, self.N, 8192)], dim=1)
            err = ((y - ref).abs().max() / ref.abs().max()).item()
            return err < 2e-2, {"rel_err": err, **self.impl_config()}

    return Int4AsymGemv


def register(run):
    """Add phases s3-s5 to the runner module `run` (bench.run) and route their cells to the ops above."""
    run.PHASES.update(phases(run.config))
    if getattr(run.GpuContext, "_paia_b200_registered", False):
        return
    base_make_op = run.GpuContext.make_op

    def make_op(self, spec):
        sh = spec["shape"]
        kw = dict(M=sh["M"], N=sh["N"], K=sh["K"], model=spec["model"], layer_name=spec["layer_name"])
        tag = self.sess_dir.parent.name                  # results/<platform_tag>/<session>
        if spec["phase"] == "s3" and spec["impl"] == "ours_fp8_w8a16":
            from bench.ops.ours_quant import OursFP8Gemv
            return OursFP8Gemv(**kw, platform_tag=tag)
        if spec["phase"] == "s4" and spec["impl"].startswith("ours_int4_"):
            from bench.ops.ours_quant import OursInt4Gemv
            return OursInt4Gemv(**kw, platform_tag=tag, mode=spec["impl"][len("ours_int4_"):])
        if spec["phase"] == "s5" and spec["impl"] == "ours_int4_asym":
            return int4_asym_op()(**kw, platform_tag=tag)
        return base_make_op(self, spec)

    run.GpuContext.make_op = make_op
    run.GpuContext._paia_b200_registered = True


def import_runner(bench_root):
    """bench.run from the harness at `bench_root` (the paia-bench directory), with this package's paia_gemv first on
    sys.path so the harness adapters load this library."""
    for p in (str(_PKG_PARENT), str(Path(bench_root).resolve())):
        if p in sys.path:
            sys.path.remove(p)
    sys.path.insert(0, str(Path(bench_root).resolve()))
    sys.path.insert(0, str(_PKG_PARENT))
    from bench import run
    register(run)
    return run


def main(argv=None):
    root = os.environ.get("PAIA_BENCH")
    if not root:
        raise SystemExit("set PAIA_BENCH to the paia-bench directory of the reference harness")
    run = import_runner(root)
    sys.argv = ["bench.run"] + list(sys.argv[1:] if argv is None else argv)
    return run.main()


if __name__ == "__main__":
    main()
