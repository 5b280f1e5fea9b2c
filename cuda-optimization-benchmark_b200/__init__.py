"""B200-native (sm_100a) kernels for the six ops of Mohamed-Alaboudi/cuda-optimization-benchmark.

The product is the C-ABI library libb200ops.so (declarations in include/b200ops.h, sources in
csrc/), whose drop-in entry points take the reference's per-task `void reference(...)` argument
lists.  This Python package builds it, binds it with ctypes and offers a torch-tensor front end
(`ops`) plus the multi-GPU helpers (`dist`).  The package directory name is not a Python
identifier; import it with importlib.import_module("cuda-optimization-benchmark_b200").
"""
from . import _build, _native, ops  # noqa: F401
from ._native import NativeLibraryError, OpError, load  # noqa: F401
