"""B200-native KV-cache manager (KCMM) for the Lattice serving stack.

The product is the native library `libkcmm.so` behind the C ABI in
`include/kcmm.h`; this package holds its sources (`csrc/`), the build step
(`build.py`) and the ctypes binding (`kcmm.py`).
"""
from .kcmm import (  # noqa: F401
    BlockLocation,
    KcmmConfig,
    KcmmError,
    KcmmLibrary,
    KcmmMetrics,
    KcmmPool,
    KcmmPoolStats,
    RopeMode,
    assert_layout,
    make_config,
)
