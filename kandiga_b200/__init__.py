"""kandiga_b200 -- B200-native (sm_100a) quantized routed-expert engine.

The CUDA kernels and the C ABI live in libkq.so (kandiga_b200/csrc, built
in-tree by kandiga_b200/build.py); this package is the thin host layer that
mirrors the reference's Python interfaces on torch CUDA tensors.
"""
from .build import LIB, build  # noqa: F401

__all__ = ["LIB", "build"]
