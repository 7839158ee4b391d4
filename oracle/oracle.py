"""ctypes binding of the C oracle (test infrastructure only).

Every function mirrors one reference function; the citations live beside the
C implementations in ``glacier_oracle.c``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libglacier_oracle.so")
_lib = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile the oracle shared library (make in oracle/)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        L = C.CDLL(_SO)
        vp, sz = C.c_void_p, C.c_size_t
        L.gor_quantize.argtypes = [vp, sz, C.c_uint32, C.c_int, vp, vp]
        L.gor_dequantize.argtypes = [vp, vp, C.c_uint32, C.c_int, sz, vp]
        L.gor_qio_payload_size.argtypes = [sz, C.c_uint32, C.c_int]
        L.gor_qio_payload_size.restype = sz
        L.gor_qio_encode.argtypes = [vp, sz, C.c_uint32, C.c_int, vp, sz]
        L.gor_qio_encode.restype = sz
        L.gor_qio_decode.argtypes = [vp, sz, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                     C.POINTER(C.c_int), vp]
        L.gor_linear_int4_f32.argtypes = [vp, sz, vp, vp, vp, vp, sz, sz, sz]
        L.gor_linear_int4_f32_mt.argtypes = [vp, sz, vp, vp, vp, vp, sz, sz, sz, sz]
        L.gor_q8_activation_group.argtypes = [sz]
        L.gor_q8_activation_group.restype = sz
        L.gor_q8_quantize_row.argtypes = [vp, sz, sz, vp, vp]
        L.gor_q8_quantize_row.restype = None
        L.gor_linear_int4_q8.argtypes = [vp, sz, vp, vp, vp, vp, sz, sz, sz]
        L.gor_linear_int4_weight_q8.argtypes = [vp, sz, vp, vp, vp, vp, sz, sz, sz]
        L.gor_rmsnorm_f32.argtypes = [vp, sz, sz, vp, C.c_float, vp]
        L.gor_rmsnorm_f32.restype = None
        L.gor_add_rmsnorm_f32.argtypes = [vp, vp, vp, sz, sz, vp, C.c_float, vp]
        L.gor_add_rmsnorm_f32.restype = None
        L.gor_silu_mul_f32.argtypes = [vp, vp, vp, sz]
        L.gor_silu_mul_f32.restype = None
        L.gor_rope_table_init.argtypes = [vp, vp, sz, sz, C.c_float]
        L.gor_rope_table_init.restype = None
        L.gor_rope_apply.argtypes = [vp, vp, sz, vp, sz, sz, sz]
        L.gor_rope_apply.restype = None
        L.gor_page_payload_offset.argtypes = [sz, C.c_int, sz, sz]
        L.gor_page_payload_offset.restype = sz
        L.gor_kv_append.argtypes = [vp, sz, vp, sz, sz, sz, vp, vp]
        L.gor_kv_append.restype = None
        L.gor_paged_attention.argtypes = [vp, vp, sz, vp, sz, sz, sz, sz, sz, vp]
        L.gor_argmax.argtypes = [vp, sz]
        L.gor_argmax.restype = sz
        L.gor_argmax_eligible.argtypes = [vp, sz, vp, sz, C.POINTER(sz), C.POINTER(sz)]
        L.gor_half_to_float.argtypes = [C.c_uint16]
        L.gor_half_to_float.restype = C.c_float
        L.gor_decode_token.argtypes = [vp, vp, sz, vp, sz, C.c_uint32, vp, vp]
        L.gor_prism_value.argtypes = [C.c_uint8, C.c_int]
        L.gor_prism_split.argtypes = [vp, sz, vp, vp, vp]
        L.gor_prism_split.restype = None
        L.gor_prism_dot_all.argtypes = [vp, vp, vp, sz, sz, vp]
        L.gor_prism_dot_all.restype = None
        L.gor_prism_dot_planes.argtypes = [vp, C.c_int, vp, vp, vp, vp, sz, sz]
        L.gor_prism_dot_planes.restype = C.c_float
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# --- quant.zig / qio.zig -------------------------------------------------------

def quantize(src, group: int, precision: int = 1):
    """quant.zig:36 quantize -> (packed uint8, scales f32)."""
    src = _f32(src).ravel()
    n = src.size
    bits = 4 if precision == 1 else 8
    packed = np.zeros((n * bits + 7) // 8, np.uint8)
    scales = np.zeros(max(1, -(-n // group)) if group else 1, np.float32)
    rc = lib().gor_quantize(_p(src), n, group, precision, _p(packed), _p(scales))
    if rc != 0:
        raise ValueError("BadGroupSize")
    return packed, scales[: -(-n // group)] if n else scales[:0]


def dequantize(packed, scales, group: int, n: int, precision: int = 1):
    """quant.zig:114 dequantize -> f32[n]."""
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = _f32(scales)
    out = np.zeros(n, np.float32)
    if lib().gor_dequantize(_p(packed), _p(scales), group, precision, n, _p(out)) != 0:
        raise ValueError("BadGroupSize")
    return out


def qio_encode(src, group: int, precision: int = 1) -> bytes:
    """qio.zig:73 encodePage."""
    src = _f32(src).ravel()
    size = lib().gor_qio_payload_size(src.size, group, precision)
    out = np.zeros(size, np.uint8)
    got = lib().gor_qio_encode(_p(src), src.size, group, precision, _p(out), size)
    if got != size:
        raise ValueError("encode failed")
    return out.tobytes()


QIO_ERRORS = {1: "TruncatedHeader", 2: "BadMagic", 3: "BadGroupSize", 4: "BadPrecision",
              5: "TruncatedScales", 6: "TruncatedPacked"}


def qio_decode(payload: bytes):
    """qio.zig:116 decodePage -> (values f32, n, group, precision)."""
    buf = np.frombuffer(payload, np.uint8).copy()
    n, g, p = C.c_uint32(), C.c_uint32(), C.c_int()
    rc = lib().gor_qio_decode(_p(buf), buf.size, C.byref(n), C.byref(g), C.byref(p), None)
    if rc:
        raise ValueError(QIO_ERRORS.get(rc, str(rc)))
    out = np.zeros(n.value, np.float32)
    lib().gor_qio_decode(_p(buf), buf.size, C.byref(n), C.byref(g), C.byref(p), _p(out))
    return out, n.value, g.value, p.value


# --- int4_matmul.zig -------------------------------------------------------------

def linear_int4(x, packed, scales, out_f: int, in_f: int, group: int, bias=None, threads: int = 1):
    """int4_matmul.zig:215 linearInt4OnTheFly (threads>1: :3046 row split)."""
    x = _f32(x).reshape(-1, in_f)
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = _f32(scales)
    bias = None if bias is None else _f32(bias)
    out = np.zeros((x.shape[0], out_f), np.float32)
    if threads > 1:
        rc = lib().gor_linear_int4_f32_mt(_p(x), x.shape[0], _p(packed), _p(scales), _p(bias),
                                          _p(out), out_f, in_f, group, threads)
    else:
        rc = lib().gor_linear_int4_f32(_p(x), x.shape[0], _p(packed), _p(scales), _p(bias),
                                       _p(out), out_f, in_f, group)
    if rc:
        raise ValueError("ShapeMismatch")
    return out


def q8_quantize(x, group: int):
    """int4_matmul.zig:365-394: one row's Q8 activation codes and per-block scales."""
    x = _f32(x).reshape(-1)
    ag = lib().gor_q8_activation_group(group)
    q = np.zeros(x.size, np.int8)
    scales = np.zeros(-(-x.size // ag), np.float32)
    lib().gor_q8_quantize_row(_p(x), x.size, group, _p(q), _p(scales))
    return q, scales


def linear_int4_q8(x, packed, scales, out_f: int, in_f: int, group: int, bias=None, weight_dispatch: bool = False):
    """int4_matmul.zig:335 linearInt4Q8OnTheFly (weight_dispatch: :422 linearInt4WeightQ8 on a
    non-AArch64 host, which sends out_f > 65536 to the FP32 path)."""
    x = _f32(x).reshape(-1, in_f)
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = _f32(scales)
    bias = None if bias is None else _f32(bias)
    out = np.zeros((x.shape[0], out_f), np.float32)
    fn = lib().gor_linear_int4_weight_q8 if weight_dispatch else lib().gor_linear_int4_q8
    if fn(_p(x), x.shape[0], _p(packed), _p(scales), _p(bias), _p(out), out_f, in_f, group):
        raise ValueError("ShapeMismatch")
    return out


# --- kernels.zig ------------------------------------------------------------------

def rmsnorm(x, weight, eps: float):
    x = _f32(x)
    x2 = x.reshape(-1, x.shape[-1])
    out = np.zeros_like(x2)
    lib().gor_rmsnorm_f32(_p(x2), x2.shape[0], x2.shape[1], _p(_f32(weight)), eps, _p(out))
    return out.reshape(x.shape)


def add_rmsnorm(a, b, weight, eps: float):
    a = _f32(a)
    b = _f32(b)
    a2, b2 = a.reshape(-1, a.shape[-1]), b.reshape(-1, a.shape[-1])
    res = np.zeros_like(a2)
    out = np.zeros_like(a2)
    lib().gor_add_rmsnorm_f32(_p(a2), _p(b2), _p(res), a2.shape[0], a2.shape[1],
                              _p(_f32(weight)), eps, _p(out))
    return res.reshape(a.shape), out.reshape(a.shape)


def silu_mul(gate, up):
    g, u = _f32(gate), _f32(up)
    out = np.zeros_like(g)
    lib().gor_silu_mul_f32(_p(g), _p(u), _p(out), g.size)
    return out


# --- RoPE --------------------------------------------------------------------------

def rope_table(positions: int, head_dim: int, theta: float):
    cos = np.zeros((positions, head_dim // 2), np.float32)
    sin = np.zeros_like(cos)
    lib().gor_rope_table_init(_p(cos), _p(sin), positions, head_dim, theta)
    return cos, sin


def rope_apply(cos, sin, row, pos: int, num_heads: int, head_dim: int):
    row = _f32(row).copy()
    lib().gor_rope_apply(_p(cos), _p(sin), cos.shape[0], _p(row), pos, num_heads, head_dim)
    return row


# --- paged KV + attention -----------------------------------------------------------

PAGE_POSITIONS = 16


def page_floats(num_layers: int, kv_dim: int) -> int:
    return num_layers * 2 * PAGE_POSITIONS * kv_dim


def page_payload_offset(layer: int, value: bool, row: int, kv_dim: int) -> int:
    return lib().gor_page_payload_offset(layer, int(value), row, kv_dim)


def kv_append(pool, pf: int, block_table, pos: int, layer: int, kv_dim: int, k, v):
    bt = np.ascontiguousarray(block_table, np.int32)
    lib().gor_kv_append(_p(pool), pf, _p(bt), pos, layer, kv_dim, _p(_f32(k)), _p(_f32(v)))


def paged_attention(q, pool, pf: int, block_table, kv_seq: int, layer: int,
                    num_heads: int, num_kv_heads: int, head_dim: int):
    q = _f32(q)
    bt = np.ascontiguousarray(block_table, np.int32)
    out = np.zeros(num_heads * head_dim, np.float32)
    rc = lib().gor_paged_attention(_p(q), _p(pool), pf, _p(bt), kv_seq, layer, num_heads,
                                   num_kv_heads, head_dim, _p(out))
    if rc:
        raise ValueError("ShapeMismatch")
    return out


# --- sampling.zig ---------------------------------------------------------------------

def argmax(v) -> int:
    v = _f32(v)
    return int(lib().gor_argmax(_p(v), v.size))


class EligibleArgmaxError(ValueError):
    pass


def argmax_eligible(logits, words):
    """sampling.zig:55 -> (token_index, eligible_rows); raises on bad mask / NaN."""
    lg = _f32(logits)
    w = np.ascontiguousarray(words, np.uint64)
    tok, rows = C.c_size_t(), C.c_size_t()
    rc = lib().gor_argmax_eligible(_p(lg), lg.size, _p(w) if w.size else None, w.size,
                                   C.byref(tok), C.byref(rows))
    if rc == 1:
        raise EligibleArgmaxError("InvalidEligibleMask")
    if rc == 2:
        raise EligibleArgmaxError("EligibleLogitNaN")
    return int(tok.value), int(rows.value)


# --- decode step ----------------------------------------------------------------------

class _Int4(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("out_f", C.c_size_t),
                ("in_f", C.c_size_t), ("group", C.c_size_t)]


class _Layer(C.Structure):
    _fields_ = [(n, _Int4) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")] + \
               [(n, C.c_void_p) for n in ("bq", "bk", "bv", "bo", "input_norm", "post_attn_norm")]


class _Model(C.Structure):
    _fields_ = [("num_layers", C.c_size_t), ("dim", C.c_size_t), ("hidden", C.c_size_t),
                ("num_heads", C.c_size_t), ("num_kv_heads", C.c_size_t), ("head_dim", C.c_size_t),
                ("vocab", C.c_size_t), ("eps", C.c_float), ("embedding_f16", C.c_void_p),
                ("final_norm", C.c_void_p), ("lm_head", _Int4), ("layers", C.POINTER(_Layer)),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("rope_positions", C.c_size_t),
                ("threads", C.c_size_t)]


class OracleModel:
    """Oracle view over a host-side synthetic model (see glacier_b200.model).

    ``m`` must expose: cfg (dict with num_layers, dim, hidden, num_heads,
    num_kv_heads, head_dim, vocab, eps), embedding (fp16 [vocab, dim]),
    final_norm, lm_head (packed, scales_f32), and layers (list of dicts with
    wq..wd as (packed, scales_f32) and bq/bk/bv, input_norm, post_attn_norm).
    """

    def __init__(self, m, rope_positions: int, threads: int = 1):
        cfg = m.cfg
        self.cfg = cfg
        self._keep = []

        def keep(a):
            self._keep.append(a)
            return a.ctypes.data

        def w(t, out_f, in_f):
            packed, scales = t
            return _Int4(keep(np.ascontiguousarray(packed, np.uint8)), keep(_f32(scales)),
                         out_f, in_f, cfg["group"])

        d, hd = cfg["dim"], cfg["head_dim"]
        qd, kvd, hid = cfg["num_heads"] * hd, cfg["num_kv_heads"] * hd, cfg["hidden"]
        layers = (_Layer * cfg["num_layers"])()
        for i, L in enumerate(m.layers):
            layers[i].wq = w(L["wq"], qd, d)
            layers[i].wk = w(L["wk"], kvd, d)
            layers[i].wv = w(L["wv"], kvd, d)
            layers[i].wo = w(L["wo"], d, qd)
            layers[i].wg = w(L["wg"], hid, d)
            layers[i].wu = w(L["wu"], hid, d)
            layers[i].wd = w(L["wd"], d, hid)
            for name in ("bq", "bk", "bv"):
                setattr(layers[i], name, keep(_f32(L[name])) if L.get(name) is not None else None)
            layers[i].bo = None
            layers[i].input_norm = keep(_f32(L["input_norm"]))
            layers[i].post_attn_norm = keep(_f32(L["post_attn_norm"]))
        self._layers = layers
        self.cos, self.sin = rope_table(rope_positions, hd, cfg["theta"])
        emb = np.ascontiguousarray(m.embedding, np.float16).view(np.uint16)
        self.s = _Model(cfg["num_layers"], d, hid, cfg["num_heads"], cfg["num_kv_heads"], hd,
                        cfg["vocab"], cfg["eps"], keep(emb), keep(_f32(m.final_norm)),
                        w(m.lm_head, cfg["vocab"], d), layers, keep(self.cos), keep(self.sin),
                        rope_positions, threads)

    def page_floats(self) -> int:
        return page_floats(self.cfg["num_layers"], self.cfg["num_kv_heads"] * self.cfg["head_dim"])

    def decode_token(self, pool, block_table, pos: int, token: int, want_logits: bool = True):
        """generate.zig:1511 forwardLayerCached over all layers + final norm + LM head."""
        bt = np.ascontiguousarray(block_table, np.int32)
        logits = np.zeros(self.cfg["vocab"], np.float32) if want_logits else None
        hidden = np.zeros(self.cfg["dim"], np.float32)
        rc = lib().gor_decode_token(C.byref(self.s), _p(pool), self.page_floats(), _p(bt), pos,
                                    token, _p(logits), _p(hidden))
        if rc:
            raise ValueError(f"decode_token failed: {rc}")
        return logits, hidden


# --- Prism progressive INT4 (progressive_int4.zig; research track) -------------------

def prism_value(nibble: int, tier: int) -> int:
    """decomposeValidNibble(...).value(tier): tier 1 coarse, 2 coarse+middle, 4 exact u - 7."""
    return int(lib().gor_prism_value(nibble, tier))


def prism_split(packed, n: int):
    """PackedPlanes.init: (coarse1, middle1, fine2) little-lane bit planes of n codes."""
    pk = np.ascontiguousarray(packed, np.uint8)
    c = np.zeros(-(-n // 8), np.uint8)
    m = np.zeros(-(-n // 8), np.uint8)
    f = np.zeros(-(-n // 4), np.uint8)
    lib().gor_prism_split(_p(pk), n, _p(c) if c.size else None, _p(m) if m.size else None,
                          _p(f) if f.size else None)
    return c, m, f


def prism_dot_all(x, packed, scales, group: int):
    """dotAll: (p1, p2, p4) dot products in one sequential pass."""
    xv = _f32(x)
    out = np.zeros(3, np.float32)
    lib().gor_prism_dot_all(_p(xv), _p(np.ascontiguousarray(packed, np.uint8)), _p(_f32(scales)), xv.size, group,
                            _p(out))
    return out


def prism_dot_planes(x, tier: int, coarse1, middle1, fine2, scales, group: int) -> float:
    """dotPlanesTier on the split planes (a tier reads only its planes)."""
    xv = _f32(x)
    arr = [None if a is None else np.ascontiguousarray(a, np.uint8) for a in (coarse1, middle1, fine2)]
    ptr = [None if a is None or a.size == 0 else _p(a) for a in arr]
    return float(lib().gor_prism_dot_planes(_p(xv), tier, ptr[0], ptr[1], ptr[2], _p(_f32(scales)), xv.size,
                                            group))
