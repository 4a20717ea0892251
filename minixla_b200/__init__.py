"""minixla_b200: a B200 (sm_100a) backend for MiniXLA's OP_FUSED hot path.

The product is the native library ``_lib/libminixla_b200.so`` (C ABI in
``include/minixla_b200.h``).  This package holds its build script, a ctypes
loader, a ctypes mirror of MiniXLA's Tensor/Node structs with the graph
constructors the hot path needs, and the seeded input generator used by the
benchmarks and tests.
"""
from . import abi, datagen
from .lib import GPU_PRECISION_3XTF32, GPU_PRECISION_TF32, load

__all__ = ["abi", "datagen", "load", "GPU_PRECISION_TF32", "GPU_PRECISION_3XTF32"]
