"""Compile-time properties of the kernels, read from ptxas's own report of the sm_100a build (build.py keeps every
object's `ptxas -v` output in paia-project_b200/build/<arch>/<source>.ptxas.txt), the B200 counterpart of the
reference's register / spill tables (src/tools/nvrtc_check.py). Every instance that a default call or an entry of
the committed tuned table resolves to has no spills and no stack frame; every TMA-fed instance with up to 8 consumer
warps is spill-free (only the rotary-epilogue instances keep a frame, for sincosf's slow path); every TMA-fed
instance's registers x threads fit the 64 K register file with one CTA per SM. Instances nothing resolves to by
default may spill: the 16-warp TMA-fed ones (held to 96 registers), the CUDA-core instances of the reference's heavy
tuples (R = 8) and some register-fed comparison kernels. Needs nvcc (the build runs here when its reports are
missing), no GPU."""
import importlib.util
import platform
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
OUT = ROOT / "paia-project_b200" / "build" / platform.machine()
TMA = re.compile(r"gemv_tma_kernelILi(\d+)ELi(\d+)ELi(\d+)ELi(\d+)ELb(\d)ELb(\d)E")


def load_reports():
    reports = sorted(OUT.glob("*.ptxas.txt"))
    if not (OUT / "tab_tma.ptxas.txt").exists():
        spec = importlib.util.spec_from_file_location("pb2_build", ROOT / "paia-project_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
        reports = sorted(OUT.glob("*.ptxas.txt"))
    rows, cur = [], None
    for f in reports:
        for line in f.read_text().splitlines():
            m = re.search(r"Compiling entry function '([^']+)'", line)
            if m:
                cur = {"fn": m.group(1), "file": f.name}
                rows.append(cur)
                continue
            m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
            if m and cur is not None:
                cur.update(stack=int(m.group(1)), spill_st=int(m.group(2)), spill_ld=int(m.group(3)))
            m = re.search(r"Used (\d+) registers", line)
            if m and cur is not None:
                cur["regs"] = int(m.group(1))
    return rows


@pytest.fixture(scope="module")
def rows():
    r = load_reports()
    assert r, "no ptxas report"
    return r


def test_every_kernel_reports_registers(rows):
    for r in rows:
        assert "regs" in r and "stack" in r, r


def test_tma_kernels_spill_only_at_16_warps(rows):
    """Every TMA-fed instance with 4 or 8 consumer warps is spill-free, and only the rotary-epilogue instances keep a
    stack frame. The 16-warp instances (576 threads) are held to 96 registers by the one-CTA-per-SM launch bound and
    spill a few bytes; the tuned table never resolves to them for a decode GEMV (test below)."""
    tma = [r for r in rows if TMA.search(r["fn"])]
    assert len(tma) >= 70, len(tma)                        # every format, decode, NC, U, PDL and the extras
    for r in tma:
        F, NC, U, DEC, BAT, ROPE = (int(v) for v in TMA.search(r["fn"]).groups())
        assert r["regs"] * (NC + 2) * 32 <= 65536, r        # one CTA of (NC + 2) warps per SM
        if NC <= 8:
            assert r["spill_st"] == 0 and r["spill_ld"] == 0, r
            assert r["stack"] == 0 or ROPE == 1, r          # the rotary epilogue's sincosf keeps a frame


FMT = {"bf16": 0, "fp8": 1, "int4": 2, "int4_asym": 3}
KEYS = {"bf16": "shapes", "fp8": "fp8_shapes", "int4": "int4_shapes", "int4_asym": "int4_asym_shapes"}
TMA_DEC = {0: 0, 1: 3, 2: 2, 3: 2}                        # the default decode of each format's TMA-fed variants
DEFAULT = {0: (2, 4, 4), 1: (2, 2, 4), 2: (4, 2, 4), 3: (4, 2, 4)}       # (R, U, W) with S = 0, H = 1
CORE_MATH = {1: 0, 2: 1, 3: 1}                             # the CUDA-core tables' math (BF16: S)


def resolve(f, N, v):
    """The kernel instance a per-format call with tuple v = (R, U, W, S, H) runs at N rows (gemv_abi.cu run():
    R = 0 -> the TMA-fed public variant; the default tuple above 1024 rows -> the TMA-fed default instance; any other
    tuple -> its CUDA-core instance gemv_kernel<F, W, R, U, math>)."""
    R, U, W, S, H = v
    if R == 0:
        return ("tma", f, W, U, TMA_DEC[f])
    if (R, U, W) == DEFAULT[f] and S == 0 and H == 1 and N > 1024:
        return ("tma", f, 8, 2, TMA_DEC[f])
    return ("core", f, W, R, U, S if f == 0 else CORE_MATH[f])


def instance_row(rows, key):
    for r in rows:
        if key[0] == "tma":
            m = TMA.search(r["fn"])
            if m and tuple(int(x) for x in m.groups()) == key[1:] + (0, 0):
                return r
        else:
            m = re.search(r"gemv_kernelILi(\d+)ELi(\d+)ELi(\d+)ELi(\d+)ELi(\d+)E", r["fn"])
            if m and "gemv_tma" not in r["fn"] and "gemv_mma" not in r["fn"] \
                    and tuple(int(x) for x in m.groups()) == key[1:]:
                return r
    return None


def test_tuned_and_default_calls_resolve_to_spill_free_instances(rows):
    """Every shape of the committed tuned table, and every format's default above 1024 rows, runs an instance with no
    spills and no stack frame."""
    import json
    table = json.loads((ROOT / "paia-project_b200" / "tuned" / "b200.json").read_text())
    checked = 0
    for kind, key in KEYS.items():
        f = FMT[kind]
        for shape, e in table.get(key, {}).items():
            N = int(shape.split("x")[0])
            v = tuple(e["variant"][k] for k in "RUWSH")
            r = instance_row(rows, resolve(f, N, v))
            assert r is not None, (kind, shape, v)
            assert r["spill_st"] == 0 and r["spill_ld"] == 0 and r["stack"] == 0, (kind, shape, v, r)
            checked += 1
        r = instance_row(rows, resolve(f, 4096, DEFAULT[f] + (0, 1)))
        assert r is not None and r["spill_st"] == 0 and r["stack"] == 0, (kind, r)
    assert checked >= 50, checked


def test_default_instances_are_lean(rows):
    """The instances a default call takes (8 consumer warps, U = 2 or 4; FP8 e4m3 decode 3, INT4 integer 2, BF16 0)
    use at most 168 registers and no stack."""
    want = {(1, 3), (2, 2), (3, 2), (0, 0)}
    seen = set()
    for r in rows:
        m = TMA.search(r["fn"])
        if not m:
            continue
        F, NC, U, DEC, BAT, ROPE = (int(v) for v in m.groups())
        if NC == 8 and (F, DEC) in want and not BAT and not ROPE:
            seen.add((F, DEC))
            assert r["regs"] <= 168 and r["stack"] == 0, r
    assert seen == want
