"""paia_gemv: B200 (sm_100a) batch-1 decode GEMV ops behind the reference's ctypes C ABI.

The op API mirrors Bejaine/PAIA-Project src/paia_gemv/__init__.py and loader.py: `load_lib()` returns a `GemvLib`
whose methods take raw device pointers (ints) and launch on torch's current CUDA stream. `quant` holds the torch
quantisers for the weight formats, `synthetic` the seeded benchmark operands.
"""
from .loader import GemvLib, load_lib  # noqa: F401
