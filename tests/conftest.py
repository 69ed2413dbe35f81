"""Test configuration: the `gpu` marker (tests that need a B200; run with `-m gpu`) and import paths for the
product package (paia-project_b200/paia_gemv) and the CPU oracle (oracle/, test infrastructure)."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "paia-project_b200"
for p in (str(PKG), str(ROOT / "oracle"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

# The reference checkout (pinning only): $PAIA_REFERENCE, else a directory named "reference" beside this repository;
# tests that need it skip where it is absent (it never exists on the GPU boxes).
REFERENCE = Path(os.environ["PAIA_REFERENCE"]) if os.environ.get("PAIA_REFERENCE") else ROOT.parent / "reference"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib_path():
    """Path of the built product library; builds it (nvcc cross-compiles, no GPU needed) if it is missing."""
    from paia_gemv import loader
    try:
        return loader.find_lib()
    except FileNotFoundError:
        import importlib.util
        spec = importlib.util.spec_from_file_location("pb2_build", PKG / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return str(mod.build())


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(ROOT / "tests" / "golden" / "golden_v1.npz")
