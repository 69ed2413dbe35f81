"""Build libpaia_gemv.so for B200 (sm_100a) in-tree.

    python paia-project_b200/build.py            # -> paia-project_b200/build/<arch>/libpaia_gemv.so
    python paia-project_b200/build.py --force    # rebuild every object

Each csrc/*.cu is compiled to an object in parallel (nvcc, -gencode arch=compute_100a,code=sm_100a, static cudart,
no torch headers), then linked into one shared library with a plain C ABI, as the reference's build.sh does
(src/paia_gemv/build.sh:8-19) but for sm_100a only. The ptxas register/spill report of every kernel is kept in
build/<arch>/ptxas_report.txt. nvcc cross-compiles, so no GPU is needed.
"""
import argparse
import os
import platform
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT = HERE / "build" / platform.machine()
LIB = OUT / "libpaia_gemv.so"
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v", "--expt-relaxed-constexpr"]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise FileNotFoundError("nvcc not found")
    return exe


def _stale(obj, deps):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force=False, verbose=False):
    OUT.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    cc = nvcc()
    jobs = []
    for s in srcs:
        obj = OUT / (s.stem + ".o")
        if force or _stale(obj, [s, *headers, Path(__file__)]):
            jobs.append((s, obj))

    def compile_one(job):
        s, obj = job
        cmd = [cc, *FLAGS, *GENCODE, "-I", str(CSRC), "-I", str(INCLUDE), "-c", str(s), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        (OUT / (s.stem + ".ptxas.txt")).write_text(r.stdout + r.stderr)
        return s, r

    failed = []
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for s, r in ex.map(compile_one, jobs):
                if r.returncode != 0:
                    failed.append((s, r))
                elif verbose:
                    print(f"compiled {s.name}")
    if failed:
        for s, r in failed:
            sys.stderr.write(f"BUILD FAILED: {s.name}\n" + "\n".join((r.stdout + r.stderr).splitlines()[:60]) + "\n")
        raise RuntimeError("nvcc failed: " + ", ".join(s.name for s, _ in failed))
    objs = [OUT / (s.stem + ".o") for s in srcs]
    if force or jobs or not LIB.exists() or _stale(LIB, objs):
        cmd = [cc, "-shared", "-cudart", "static", *GENCODE, *map(str, objs), "-o", str(LIB)]
        subprocess.run(cmd, check=True)
        with open(OUT / "ptxas_report.txt", "w") as f:
            for s in srcs:
                p = OUT / (s.stem + ".ptxas.txt")
                if p.exists():
                    f.write(p.read_text())
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True))
