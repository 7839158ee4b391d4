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
    def __init__(self, code: int, msg: str, reason: int = 0):
        super().__init__(f"glacier_cuda error {code}: {msg}")
        self.code = code
        self.reason = reason  # enum glacier_cuda_format_reason when code is EFORMAT


EINVAL, ECUDA, ENOMEM, EMASK, ENAN, EUNSUPPORTED, EFORMAT = -1, -2, -3, -4, -5, -6, -7

vp, sz, i32, u32, f32 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_float


class ArgmaxResult(C.Structure):
    """glacier_argmax_result (24 bytes, same layout as int4_neon.c:8-19)."""
    _fields_ = [("value", C.c_float), ("index", C.c_size_t), ("valid", C.c_int), ("saw_nan", C.c_int)]


# name -> (argtypes, restype); the single source of the Python-side signatures.
SIGNATURES = {
    "glacier_cuda_last_error": ([], C.c_char_p),
    "glacier_cuda_version": ([], i32),
    "glacier_cuda_device_status": ([i32], i32),
    "glacier_cuda_launch_count": ([], C.c_ulonglong),
    "glacier_cuda_int4_matvec_f32": ([vp, vp, vp, vp, vp, sz, sz, sz, vp], i32),
    "glacier_cuda_int4_matvec_f16scale": ([vp, vp, vp, vp, vp, sz, sz, sz, vp], i32),
    "glacier_cuda_int4_linear": ([vp, sz, vp, vp, i32, vp, vp, sz, sz, sz, vp], i32),
    "glacier_cuda_int4_linear_q8": ([vp, sz, vp, vp, i32, vp, vp, sz, sz, sz, vp], i32),
    "glacier_cuda_int4_matmul_workspace": ([sz, sz, sz], sz),
    "glacier_cuda_int4_matmul_f16scale": ([vp, sz, vp, vp, vp, vp, sz, sz, sz, vp, sz, vp], i32),
    "glacier_cuda_rmsnorm_f32": ([vp, vp, f32, vp, sz, sz, vp], i32),
    "glacier_cuda_add_rmsnorm_f32": ([vp, vp, vp, vp, f32, vp, sz, sz, vp], i32),
    "glacier_cuda_silu_mul_f32": ([vp, vp, sz, vp, sz, sz, sz, vp], i32),
    "glacier_cuda_embedding_f16": ([vp, sz, sz, vp, sz, vp, vp], i32),
    "glacier_cuda_qkv_rope_append_f32": ([vp, sz, vp, vp, vp, sz, vp, sz, sz, sz, sz, vp, sz, vp, sz, vp, sz,
                                          sz, vp], i32),
    "glacier_cuda_paged_attention_workspace": ([sz, sz, sz, sz, sz], sz),
    "glacier_cuda_paged_attention_f32": ([vp, vp, sz, vp, sz, vp, sz, sz, sz, sz, sz, sz, vp, vp, sz, vp], i32),
    "glacier_cuda_argmax_workspace": ([sz, sz], sz),
    "glacier_cuda_argmax_eligible_f32": ([vp, sz, sz, vp, sz, vp, vp, vp, vp, sz, vp], i32),
    "glacier_cuda_argmax_eligible_f32_noalloc": ([vp, sz, sz, vp, sz, vp, vp, vp, vp], i32),
    "glacier_cuda_model_create": ([vp], vp),
    "glacier_cuda_model_destroy": ([vp], None),
    "glacier_cuda_model_load_int4": ([vp, i32, i32, vp, sz, vp, sz], i32),
    "glacier_cuda_model_load_int4_rows4": ([vp, i32, i32, vp, sz, vp, sz], i32),
    "glacier_cuda_model_load_pair_nibble": ([vp, i32, vp, sz, vp, sz], i32),
    "glacier_cuda_model_load_qio": ([vp, i32, i32, vp, sz], i32),
    "glacier_cuda_model_load_f32": ([vp, i32, i32, vp, sz], i32),
    "glacier_cuda_model_load_embedding_f16": ([vp, vp, sz], i32),
    "glacier_cuda_model_load_embedding_f32": ([vp, vp, sz], i32),
    "glacier_cuda_format_error": ([], C.c_int32),
    "glacier_cuda_crc32": ([vp, sz], C.c_uint32),
    "glacier_cuda_glacier_open": ([vp, C.c_uint64, vp], i32),
    "glacier_cuda_glacier_validate_pages": ([vp, C.c_uint64], i32),
    "glacier_cuda_glacier_page": ([vp, C.c_uint64, C.c_uint64, vp], i32),
    "glacier_cuda_glacier_pages": ([vp, C.c_uint64, vp, C.c_uint64, vp], i32),
    "glacier_cuda_glacier_page_decode_f32": ([vp, C.c_uint64, C.c_uint64, vp, C.c_uint64], i32),
    "glacier_cuda_glacier_geometry": ([vp, C.c_uint64, vp], i32),
    "glacier_cuda_model_load_glacier": ([vp, vp, C.c_uint64, i32], i32),
    "glacier_cuda_context_create": ([i32], vp),
    "glacier_cuda_context_destroy": ([vp], None),
    "glacier_cuda_context_stream": ([vp], vp),
    "glacier_cuda_int4_weight_create": ([vp, vp, C.c_uint64, vp, C.c_uint64, u32, u32, u32], vp),
    "glacier_cuda_int4_weight_create_ex": ([vp, vp, C.c_uint64, vp, C.c_uint64, u32, u32, u32, u32], vp),
    "glacier_cuda_int4_weight_destroy": ([vp], None),
    "glacier_cuda_int4_matvec_dispatch": ([vp, vp, vp, C.c_uint64, vp, C.c_uint64], i32),
    "glacier_cuda_int4_weight_read_output": ([vp, vp, C.c_uint64], i32),
    "glacier_cuda_int4_weight_matvec": ([vp, vp, vp, vp, vp], i32),
    "glacier_cuda_int4_weight_matmul": ([vp, vp, sz, vp, sz, sz, vp, vp], i32),
    "glacier_cuda_int4_weight_lmhead_argmax": ([vp, vp, sz, vp, sz, vp, vp, vp, vp, vp], i32),
    "glacier_cuda_all_finite_f32": ([vp, sz, vp, vp], i32),
    "glacier_cuda_glrt_open": ([vp, C.c_uint64, vp, vp], i32),
    "glacier_cuda_glrt_record": ([vp, C.c_uint64, C.c_uint64, vp], i32),
    "glacier_cuda_glrt_records": ([vp, C.c_uint64, vp, C.c_uint64, vp], i32),
    "glacier_cuda_glrt_model_info": ([vp, C.c_uint64, vp, vp], i32),
    "glacier_cuda_model_load_glrt": ([vp, vp, C.c_uint64, vp], i32),
    "glacier_cuda_rows4_k16_to_row_major": ([vp, vp, sz, sz], i32),
    "glacier_cuda_rows4_scales_to_row_major": ([vp, vp, sz, sz], i32),
    "glacier_cuda_pair_nibble_split": ([vp, vp, sz, sz, sz, vp, vp, vp, vp], i32),
    "glacier_cuda_model_finalize": ([vp], i32),
    "glacier_cuda_model_reserve": ([vp, sz, sz], i32),
    "glacier_cuda_kv_create": ([vp, sz], vp),
    "glacier_cuda_kv_destroy": ([vp], None),
    "glacier_cuda_kv_pages": ([vp], vp),
    "glacier_cuda_kv_page_floats": ([vp], sz),
    "glacier_cuda_decode_step": ([vp, vp, sz, vp, vp, vp, sz, vp, sz, vp, vp, vp, vp], i32),
    "glacier_cuda_prefill": ([vp, vp, vp, sz, i32, vp, sz, vp, sz, vp, vp, vp, vp], i32),
    "glacier_cuda_tp_unique_id": ([vp], i32),
    "glacier_cuda_model_tp_init": ([vp, C.c_int, C.c_int, vp], i32),
    "glacier_cuda_model_tp_lanes": ([vp, C.c_int, C.c_int], i32),
    "glacier_cuda_model_profile": ([vp, C.c_int], i32),
    "glacier_cuda_model_profile_read": ([vp, vp, vp, sz], i32),
    "glacier_cuda_model_persistent": ([vp, C.c_int], i32),
}

# enum glacier_cuda_tensor_kind
W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_LM_HEAD, B_Q, B_K, B_V, N_INPUT, N_POST_ATTN, N_FINAL = range(14)


class FileInfo(C.Structure):
    """glacier_cuda_file_info."""
    _fields_ = [(n, C.c_uint64) for n in ("container_bytes", "meta_offset", "meta_len", "num_pages",
                                          "page_index_offset", "page_data_offset")]


class PageEntry(C.Structure):
    """glacier_cuda_page_entry: one decoded 64-byte page index entry."""
    _fields_ = [("page_id", C.c_uint64), ("layer_idx", C.c_uint32), ("tensor_kind", C.c_uint32),
                ("row_start", C.c_uint64), ("row_end", C.c_uint64), ("precision", C.c_uint8),
                ("quant_group", C.c_uint8), ("reserved", C.c_uint16), ("crc32", C.c_uint32),
                ("data_offset", C.c_uint64), ("data_len", C.c_uint64)]


class FileGeometry(C.Structure):
    """glacier_cuda_file_geometry."""
    _fields_ = [(n, C.c_uint32) for n in ("num_layers", "dim", "hidden", "vocab", "group_size", "has_lm_head",
                                          "has_qkv_bias")]


class GlrtOptions(C.Structure):
    """glacier_cuda_glrt_options."""
    _fields_ = [("skip_payload_crc", C.c_uint32), ("skip_payload_digest", C.c_uint32), ("reject_v1", C.c_uint32),
                ("abi_policy", C.c_uint32), ("expected_source_fingerprint", C.c_void_p)]


class GlrtInfo(C.Structure):
    """glacier_cuda_glrt_info."""
    _fields_ = [("version", C.c_uint32), ("abi_policy", C.c_uint32), ("record_count", C.c_uint64),
                ("data_offset", C.c_uint64), ("file_size", C.c_uint64),
                ("source_fingerprint", C.c_uint8 * 32), ("abi_fingerprint", C.c_uint8 * 32)] + \
               [(n, C.c_uint32) for n in ("dim", "hidden", "num_layers", "vocab", "num_heads", "head_dim",
                                          "num_kv_heads", "tie_embeddings")] + \
               [("rms_eps", C.c_float), ("rope_theta", C.c_float), ("mlp_layout", C.c_uint32),
                ("group_size", C.c_uint32)]


class GlrtEntry(C.Structure):
    """glacier_cuda_glrt_entry: one decoded runtime-image record."""
    _fields_ = [("layer_idx", C.c_uint32), ("tensor_kind", C.c_uint32), ("encoding", C.c_uint16),
                ("packed_layout", C.c_uint16), ("role", C.c_uint16), ("pair_nibble_layout", C.c_uint16),
                ("group_size", C.c_uint32), ("out_f", C.c_uint32), ("in_f", C.c_uint32),
                ("payload_crc32", C.c_uint32), ("num_elements", C.c_uint64),
                ("stream_offset", C.c_uint64 * 5), ("stream_len", C.c_uint64 * 5),
                ("payload_digest", C.c_uint8 * 32)]


class ModelConfigC(C.Structure):
    """glacier_cuda_model_config."""
    _fields_ = [(n, C.c_uint32) for n in ("num_layers", "dim", "hidden", "num_heads", "num_kv_heads",
                                          "head_dim", "vocab", "group_size")] + \
               [("rms_eps", C.c_float), ("rope_theta", C.c_float), ("max_positions", C.c_uint32),
                ("scales_f16", C.c_uint32)]


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
        reason = lib().glacier_cuda_format_error() if rc == EFORMAT else 0
        raise GlacierCudaError(rc, msg.decode() if msg else "", reason)
    return rc


def call(name: str, *args) -> int:
    return check(getattr(lib(), name)(*args))


def handle(ptr):
    """Raise with the library's message when a handle-returning call gave NULL."""
    if not ptr:
        msg = lib().glacier_cuda_last_error()
        raise GlacierCudaError(EINVAL, msg.decode() if msg else "NULL handle")
    return ptr
