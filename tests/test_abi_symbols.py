"""The C-ABI library loads on a CPU-only host and exports every declared symbol."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "glacier_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(glacier_cuda_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "glacier_cuda_int4_matvec_f32" in names and len(names) >= 5


def test_library_exports_every_declared_symbol():
    from glacier_b200 import _lib
    so = ctypes.CDLL(_lib.LIB_PATH)  # loads without a GPU: no CUDA call at load time
    missing = [n for n in declared_functions() if not hasattr(so, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from glacier_b200 import _lib
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_version_callable_without_gpu():
    from glacier_b200 import _lib
    assert _lib.lib().glacier_cuda_version() >= 1


def test_context_create_without_gpu_returns_null():
    """On a host with no usable GPU the context constructor fails cleanly (NULL + message)."""
    import torch
    if torch.cuda.is_available():
        return
    from glacier_b200 import _lib
    L = _lib.lib()
    assert not L.glacier_cuda_context_create(0)
    assert b"context_create" in L.glacier_cuda_last_error()
