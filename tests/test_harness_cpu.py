"""Harness integration without a GPU: the reference's unchanged cell runner (paia-bench bench.run, found through
$PAIA_BENCH or the reference checkout) gains phases s3-s5 from paia_gemv.harness.register, their cells follow the
runner's field layout and the formats' K rules, and GpuContext.make_op builds the right adapter for every cell (the
reference's own FP8 / INT4 adapters, loading this library, and the asymmetric INT4 op). Skipped where the reference
harness is not present (it does not travel to the GPU box)."""
import os
import sys
from pathlib import Path

import pytest


def _bench_root():
    from conftest import REFERENCE
    for cand in (os.environ.get("PAIA_BENCH"), str(REFERENCE / "paia-bench")):
        if cand and (Path(cand) / "bench" / "run.py").exists():
            return cand
    return None


ROOT = _bench_root()
pytestmark = pytest.mark.skipif(ROOT is None, reason="reference harness (paia-bench) not present")


@pytest.fixture(scope="module")
def run():
    saved = list(sys.path)
    mods = {k: v for k, v in sys.modules.items() if k == "bench" or k.startswith("bench.")}
    for k in mods:
        del sys.modules[k]
    from paia_gemv import harness
    r = harness.import_runner(ROOT)
    yield r
    for k in [k for k in sys.modules if k == "bench" or k.startswith("bench.")]:
        del sys.modules[k]
    sys.modules.update(mods)
    sys.path[:] = saved


def test_phases_registered_and_cells_well_formed(run):
    for ph in ("s3", "s4", "s5"):
        assert ph in run.PHASES
    cfg = run.config.shapes_cfg()
    s3, s4, s5 = run.PHASES["s3"](), run.PHASES["s4"](), run.PHASES["s5"]()
    keys = {"phase", "op", "impl", "precision", "hot_or_cold", "shape", "model", "layer_name", "timing_mode"}
    for cells, kmult in ((s3, 16), (s4, 128), (s5, 128)):
        assert cells and all(set(c) == keys for c in cells)
        assert all(c["shape"]["M"] == 1 and c["shape"]["K"] % kmult == 0 for c in cells)
    # every model shape whose K the format accepts, in every timing mode
    n_models = sum(1 for m in cfg["models"].values() for (_, k) in m["shapes"].values() if k % 16 == 0)
    assert sum(1 for c in s3 if c["model"] != "synthetic") == 3 * n_models
    assert {c["impl"] for c in s4} == {"ours_int4_fused", "ours_int4_naive", "ours_int4_unfused"}
    assert all(c["timing_mode"] == "graph" for c in s4 if c["impl"] != "ours_int4_fused")
    assert len({run.cell_id(c) for c in s3 + s4 + s5}) == len(s3) + len(s4) + len(s5)


def test_make_op_builds_the_adapters(run):
    ctx = run.GpuContext.__new__(run.GpuContext)           # no device needed to construct the ops
    ctx.sess_dir = Path("results") / "b200" / "debug_cpu"
    seen = {}
    for ph in ("s3", "s4", "s5"):
        for c in run.PHASES[ph]():
            if c["model"] == "llama31_8b" and c["layer_name"] == "gate_up_fused":
                op = ctx.make_op(c)
                seen[c["impl"]] = op
                sh = c["shape"]
                assert (op.M, op.N, op.K) == (sh["M"], sh["N"], sh["K"])
                assert sum(op.bytes().values()) > 0 and op.footprint_bytes() > 0
    assert type(seen["ours_fp8_w8a16"]).__name__ == "OursFP8Gemv"
    assert type(seen["ours_int4_fused"]).__name__ == "OursInt4Gemv" and seen["ours_int4_naive"].mode == "naive"
    a = seen["ours_int4_asym"]
    assert type(a).__name__ == "Int4AsymGemv"
    N, K = 28672, 4096
    assert a.bytes() == {"weights": N * K // 2, "metadata": 4 * N * (K // 128), "act_in": 2 * K, "out": 2 * N}
    # the adapters load this library (the reference loader's search order is not involved)
    from paia_gemv import loader
    assert seen["ours_fp8_w8a16"].lib.path == loader.find_lib()


def test_other_phases_still_route_to_the_runner(run):
    ctx = run.GpuContext.__new__(run.GpuContext)
    ctx.sess_dir = Path("results") / "b200" / "debug_cpu"
    with pytest.raises(ValueError, match="no op for"):
        ctx.make_op({"phase": "zz", "impl": "none", "shape": {"M": 1, "N": 8, "K": 8}, "model": None,
                     "layer_name": None})
