"""KERNIX-B200: the KERNIX .knx model forward path (load + forward) as a B200-native (sm_100a) library.

The product is libkernix.so (host C runtime + CUDA kernels, C-ABI in include/*.h). This package holds the
numpy/ctypes binding `Model` (same interface as the reference's python/kernix.py), the build script, a torch-free
.knx writer and the seeded benchmark configurations.
"""
from .kernix import Model, lib  # noqa: F401

__all__ = ["Model", "lib"]
