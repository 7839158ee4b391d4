"""Glacier B200: INT4 decode hot path of Glacier Engine as sm_100a CUDA kernels.

The compute lives in ``libglacier_cuda.so`` (C ABI, ``include/glacier_cuda.h``).
This package holds the host-side mirror of the reference's operator API for
tests and benchmarks: ctypes bindings (``_lib``), reference-named operator
wrappers over device tensors (``ops``) and the synthetic-model / decode driver
(``model``).
"""
from ._lib import GlacierCudaError, LIB_PATH, lib  # noqa: F401
