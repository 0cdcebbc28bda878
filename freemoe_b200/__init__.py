"""freemoe_b200: B200 (sm_100a) backend for FreeMoe's routed-expert MoE hot path.

The product is the C ABI in ``include/freemoe_b200.h``, implemented by
``libfreemoe_b200.so`` (hand-written CUDA in ``csrc/``), and the C++17
``fm::Backend`` adapter in ``backend/``.  This Python package only binds the
C ABI for tests and the benchmark.
"""
from ._lib import (GEOMETRY, ORDER_ANY, ORDER_AVX2, ORDER_SCALAR, TYPE_F32, TYPE_Q4_K, TYPE_Q8_0,
                   X_BF16, X_F32, FmError, LIB_PATH, SIGNATURES, load)

__all__ = [
    "GEOMETRY", "ORDER_ANY", "ORDER_AVX2", "ORDER_SCALAR", "TYPE_F32", "TYPE_Q4_K", "TYPE_Q8_0",
    "X_BF16", "X_F32", "FmError", "LIB_PATH", "SIGNATURES", "load",
]
