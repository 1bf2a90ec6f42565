"""Python side of the B200-native Opure-VoxelEngine decode path.

The compute path is native: libopure_cuda.so (sm_100a kernels behind the C ABI in
include/opure_cuda.h) and libopure_engine.so (the C++20 host engine, include/opure_engine.h).
This package only binds them with ctypes; it never computes on the CPU.
"""
from . import cuda  # noqa: F401

__all__ = ["cuda"]
