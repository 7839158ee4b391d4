"""Generate the golden fixtures that pin the CPU oracle.

Usage:  python tests/golden/make_golden.py <path-to-glacier-engine-checkout>

Two fixture files are written next to this script:

* ``layer0_numpy.npz`` -- outputs of the reference's own Python float reference
  (``tools/reference_layer0.py``: ``rmsnorm``, ``silu``, ``softmax`` and the
  cos/sin tables of its NeoX ``rope``), imported from the checkout and evaluated on seeded inputs.
* ``int4_formula.json`` -- the deterministic weight/input formulas of the
  reference's INT4 kernel microbench (``bench/int4_kernel.zig:38-43,77-81``),
  quantized by an independent vectorised numpy restatement of
  ``src/core/quant.zig:36-111`` and multiplied in float64.  Only digests of the
  packed bytes and scales are stored (the matrix is regenerated from the
  formula), plus the float64 product rounded to float32.

The checkout is read only at generation time; the tests use the committed
fixtures and never need the reference.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def formula_weights(out_f: int, in_f: int) -> np.ndarray:
    """bench/int4_kernel.zig:38-43: ((i*29+7) % 101 - 50) / 127 over the flat index."""
    i = np.arange(out_f * in_f, dtype=np.int64)
    return (((i * 29 + 7) % 101).astype(np.float32) - np.float32(50)) / np.float32(127)


def formula_input(in_f: int) -> np.ndarray:
    """bench/int4_kernel.zig:77-81: ((i*13+3) % 47 - 23) / 31."""
    i = np.arange(in_f, dtype=np.int64)
    return (((i * 13 + 3) % 47).astype(np.float32) - np.float32(23)) / np.float32(31)


def numpy_quantize_int4(src: np.ndarray, group: int):
    """Vectorised restatement of src/core/quant.zig:36-111 for INT4, n % group == 0."""
    g = src.reshape(-1, group).astype(np.float32)
    qmax = 8 if group >= 16 else 7
    mn = np.minimum(g.min(axis=1), np.float32(0))
    mx = np.maximum(g.max(axis=1), np.float32(0))
    scale = np.maximum(-mn / np.float32(7), mx / np.float32(qmax)).astype(np.float32)
    inv = np.where(scale == 0, np.float32(0), np.float32(1) / np.where(scale == 0, 1, scale))
    inv = inv.astype(np.float32)
    t = (g * inv[:, None]).astype(np.float32)
    # Round half away from zero (Zig @round) without the float32 (|t| + 0.5)
    # double rounding: compare the exact fractional part with one half.
    a = np.abs(t)
    r = np.floor(a)
    q = np.sign(t) * (r + (a - r >= np.float32(0.5)))
    q = np.clip(q, -7, qmax).astype(np.int32) + 7
    codes = q.reshape(-1).astype(np.uint8)
    packed = (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8)
    return packed, scale


def numpy_dequantize_int4(packed: np.ndarray, scales: np.ndarray, group: int) -> np.ndarray:
    codes = np.empty(packed.size * 2, np.int32)
    codes[0::2] = packed & 0x0F
    codes[1::2] = packed >> 4
    return (codes - 7).reshape(-1, group).astype(np.float64) * scales[:, None].astype(np.float64)


def load_reference_layer0(checkout: str):
    path = os.path.join(checkout, "tools", "reference_layer0.py")
    spec = importlib.util.spec_from_file_location("reference_layer0", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_layer0(ref) -> None:
    rng = np.random.default_rng(20240601)
    dim, seq, hidden = 64, 5, 96
    x = rng.standard_normal((seq, dim), dtype=np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    eps = np.float32(1e-6)
    rms = ref.rmsnorm(x, w, eps).astype(np.float32)
    gate = rng.standard_normal((seq, hidden), dtype=np.float32)
    up = rng.standard_normal((seq, hidden), dtype=np.float32)
    swiglu = (ref.silu(gate) * up).astype(np.float32)
    # reference_layer0.rope rebinds x0 through a numpy view, so its second
    # output uses the already-rotated first one; it is therefore used only to
    # read the cos/sin tables: rope(e_k) returns cos in slot k, and rope(e_{k+half})
    # returns -sin in slot k.
    positions, table_dim = 9, 32
    half = table_dim // 2
    ones_lo = np.zeros((positions, table_dim), np.float32)
    ones_lo[:, :half] = 1
    ones_hi = np.zeros((positions, table_dim), np.float32)
    ones_hi[:, half:] = 1
    rope_cos = ref.rope(ones_lo, 1, table_dim, theta=1000000.0)[:, :half].astype(np.float32)
    rope_sin = -ref.rope(ones_hi, 1, table_dim, theta=1000000.0)[:, :half].astype(np.float32)
    scores = rng.standard_normal((3, 37), dtype=np.float32) * np.float32(4)
    probs = ref.softmax(scores).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "layer0_numpy.npz"), x=x, w=w, eps=eps, rms=rms,
                        gate=gate, up=up, swiglu=swiglu, rope_cos=rope_cos, rope_sin=rope_sin,
                        table_dim=table_dim, theta=np.float32(1e6),
                        scores=scores, probs=probs)


def make_formula() -> None:
    out = {}
    for out_f, in_f, group in ((4864, 896, 8), (4864, 896, 32), (37, 64, 8)):
        w = formula_weights(out_f, in_f)
        x = formula_input(in_f)
        packed, scales = numpy_quantize_int4(w, group)
        y = (numpy_dequantize_int4(packed, scales, group).reshape(out_f, in_f)
             @ x.astype(np.float64)).astype(np.float32)
        out[f"{out_f}x{in_f}_g{group}"] = {
            "out_f": out_f, "in_f": in_f, "group": group,
            "packed_sha256": hashlib.sha256(packed.tobytes()).hexdigest(),
            "scales_sha256": hashlib.sha256(scales.astype("<f4").tobytes()).hexdigest(),
            "y": [float(v) for v in y],
        }
    with open(os.path.join(HERE, "int4_formula.json"), "w") as f:
        json.dump(out, f)


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    make_layer0(load_reference_layer0(sys.argv[1]))
    make_formula()


if __name__ == "__main__":
    main()
