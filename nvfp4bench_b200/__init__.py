"""nvfp4bench_b200 - B200-native (sm_100a) NVFP4 block-scaled GEMM engine.

The product is the in-tree shared library lib/libnvfp4_b200.so (hand-written tcgen05 CUDA
kernels behind the C ABI in include/nvfp4_b200.h) and the C++ harness bin/nvfp4bench.
This Python package is a thin ctypes binding over that C ABI (``api``) and the build
recipe (``build``).
"""
from . import build  # noqa: F401

__all__ = ["build", "api"]


def __getattr__(name):
    if name == "api":
        import importlib
        return importlib.import_module(".api", __name__)
    raise AttributeError(name)
