"""ctypes loader for libglacier_cuda.so (the in-tree C-ABI library).

The library is the product; this module only binds its entry points.  It never
falls back to another implementation: if the shared object is missing or a call
fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libglacier_cuda.so")

_lib = None


class GlacierCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"glacier_cuda error {code}: {msg}")
        self.code = code


EINVAL, ECUDA, ENOMEM, EMASK, ENAN, EUNSUPPORTED = -1, -2, -3, -4, -5, -6

vp, sz, i32, u32, f32 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_float


class ArgmaxResult(C.Structure):
    """glacier_argmax_result (24 bytes, same layout as int4_neon.c:8-19)."""
    _fields_ = [("value", C.c_float), ("index", C.c_size_t), ("valid", C.c_int), ("saw_nan", C.c_int)]


# name -> (argtypes, restype); the single source of the Python-side signatures.
SIGNATURES = {
    "glacier_cuda_last_error": ([], C.c_char_p),
    "glacier_cuda_version": ([], i32),
    "glacier_cuda_device_status": ([i32], i32),
    "glacier_cuda_int4_matvec_f32": ([vp, vp, vp, vp, vp, sz, sz, sz, vp], i32),
    "glacier_cuda_int4_matvec_f16scale": ([vp, vp, vp, vp, vp, sz, sz, sz, vp], i32),
    "glacier_cuda_int4_linear": ([vp, sz, vp, vp, i32, vp, vp, sz, sz, sz, vp], i32),
}


def lib():
    """Load and bind the library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with python glacier-engine_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc: int) -> int:
    if rc != 0:
        msg = lib().glacier_cuda_last_error()
        raise GlacierCudaError(rc, msg.decode() if msg else "")
    return rc


def call(name: str, *args) -> int:
    return check(getattr(lib(), name)(*args))
