"""Glacier B200: INT4 decode hot path of Glacier Engine as sm_100a CUDA kernels.

The compute lives in ``libglacier_cuda.so`` (C ABI, ``include/glacier_cuda.h``).
This package holds the host-side mirror of the reference's operator API for
tests and benchmarks: ctypes bindings (``_lib``), reference-named operator
wrappers over device tensors (``ops``), the synthetic-model / decode driver
(``model``), and the model-file readers and loaders for the portable
``.glacier`` container (``glacier_file``) and the prepared ``.glrt`` runtime
image (``runtime_image``).
"""
from ._lib import GlacierCudaError, LIB_PATH, lib  # noqa: F401
