"""Pins the CPU oracle against the reference's own known answers and fixtures.

The known-answer cases are the literals of the reference's unit tests (cited
per test); the fixtures in tests/golden/ come from the reference's Python float
reference and from an independent numpy restatement of its quantizer
(tests/golden/make_golden.py).  No GPU needed.
"""
import hashlib
import json
import math
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# --- src/core/quant.zig tests ------------------------------------------------------

def test_int4_packs_two_per_byte_zero_is_0x77():
    # quant.zig:223-235
    packed, scales = oracle.quantize(np.zeros(4, np.float32), 4)
    assert packed.tolist() == [0x77, 0x77]


def test_int4_group16_full_positive_code_group8_compatible():
    # quant.zig:237-255
    src = np.zeros(16, np.float32)
    src[0] = 1
    packed, scales = oracle.quantize(src, 16)
    assert packed[0] == 0x7F and scales[0] == np.float32(0.125)
    packed8, _ = oracle.quantize(src[:8], 8)
    assert packed8[0] == 0x7E


def test_zero_tensor_zero_scales():
    # quant.zig:278-296
    packed, scales = oracle.quantize(np.zeros(8, np.float32), 4)
    assert scales.tolist() == [0.0, 0.0]
    back = oracle.dequantize(packed, scales, 4, 8)
    assert (back == 0).all()


def test_independent_group_scales():
    # quant.zig:298-313
    src = np.concatenate([np.arange(8) * 0.001, np.arange(8) * 10.0]).astype(np.float32)
    _, scales = oracle.quantize(src, 8)
    assert scales.size == 2 and scales[0] < scales[1] / 1000


def test_int8_round_trip_integers():
    # quant.zig:209-221
    src = np.array([0, 1, -1, 2, -2, 64, -64, 127, -127], np.float32)
    packed, scales = oracle.quantize(src, 16, precision=0)
    back = oracle.dequantize(packed, scales, 16, src.size, precision=0)
    assert np.abs(back - src).max() <= 1.0


def test_nibble_codes_decode_to_signed_values():
    # int4_weights.zig:449-461: {0x80, 0x0f} -> {-7, 1, 8, -7}
    back = oracle.dequantize(np.array([0x80, 0x0F], np.uint8), np.array([1.0], np.float32), 4, 4)
    assert back.tolist() == [-7.0, 1.0, 8.0, -7.0]


# --- src/model/qio.zig tests ---------------------------------------------------------

def test_qio_round_trip_and_header():
    # qio.zig:172-196
    rng = np.random.default_rng(7)
    src = ((rng.random(128, dtype=np.float32) * 2 - 1) * 0.5).astype(np.float32)
    payload = oracle.qio_encode(src, 32)
    assert int.from_bytes(payload[:4], "little") == 0x514F4954
    back, n, g, p = oracle.qio_decode(payload)
    assert (n, g, p) == (128, 32, 1)
    assert np.abs(back - src).max() < 0.06


def test_qio_rejects_bad_payloads():
    # qio.zig:205-225
    with pytest.raises(ValueError, match="BadMagic"):
        oracle.qio_decode(bytes(16))
    hdr = bytearray(16)
    hdr[:4] = (0x514F4954).to_bytes(4, "little")
    with pytest.raises(ValueError, match="BadGroupSize"):
        oracle.qio_decode(bytes(hdr))
    enc = oracle.qio_encode(np.ones(8, np.float32), 4)
    with pytest.raises(ValueError, match="TruncatedPacked"):
        oracle.qio_decode(enc[:-1])
    with pytest.raises(ValueError, match="TruncatedHeader"):
        oracle.qio_decode(enc[:8])


# --- INT4 matvec against the microbench formula fixture ---------------------------------

def _formula(out_f, in_f):
    i = np.arange(out_f * in_f, dtype=np.int64)
    w = (((i * 29 + 7) % 101).astype(np.float32) - np.float32(50)) / np.float32(127)
    j = np.arange(in_f, dtype=np.int64)
    x = (((j * 13 + 3) % 47).astype(np.float32) - np.float32(23)) / np.float32(31)
    return w, x


@pytest.mark.parametrize("key", ["4864x896_g8", "4864x896_g32", "37x64_g8"])
def test_formula_quantize_and_matvec(key):
    fx = json.load(open(os.path.join(GOLDEN, "int4_formula.json")))[key]
    w, x = _formula(fx["out_f"], fx["in_f"])
    packed, scales = oracle.quantize(w, fx["group"])
    assert hashlib.sha256(packed.tobytes()).hexdigest() == fx["packed_sha256"]
    assert hashlib.sha256(scales.astype("<f4").tobytes()).hexdigest() == fx["scales_sha256"]
    y = oracle.linear_int4(x, packed, scales, fx["out_f"], fx["in_f"], fx["group"])[0]
    ref = np.array(fx["y"], np.float32)
    # float64 product vs the reference's fp32 Vec8 accumulation order.
    assert np.abs(y - ref).max() <= 2e-5 * max(1.0, np.abs(ref).max())


def test_threaded_row_split_is_bit_identical():
    # int4_matmul.zig:3601 "parallel split is bit-identical"
    w, x = _formula(4864, 896)
    packed, scales = oracle.quantize(w, 32)
    a = oracle.linear_int4(x, packed, scales, 4864, 896, 32)
    b = oracle.linear_int4(x, packed, scales, 4864, 896, 32, threads=7)
    assert a.tobytes() == b.tobytes()


def test_generic_path_odd_group_matches_dequant():
    # int4_matmul.zig:283-300 generic path: groups crossing rows (in_f % group != 0).
    rng = np.random.default_rng(3)
    out_f, in_f, group = 5, 20, 12
    w = rng.standard_normal(out_f * in_f).astype(np.float32)
    packed, scales = oracle.quantize(w, group)
    deq = oracle.dequantize(packed, scales, group, out_f * in_f).reshape(out_f, in_f)
    x = rng.standard_normal(in_f).astype(np.float32)
    bias = rng.standard_normal(out_f).astype(np.float32)
    y = oracle.linear_int4(x, packed, scales, out_f, in_f, group, bias=bias)[0]
    assert np.abs(y - (deq.astype(np.float64) @ x + bias)).max() < 2e-5


# --- kernels.zig / RoPE / softmax against reference_layer0.py -------------------------

def test_layer0_fixture_norm_swiglu_rope_softmax():
    fx = np.load(os.path.join(GOLDEN, "layer0_numpy.npz"))
    rms = oracle.rmsnorm(fx["x"], fx["w"], float(fx["eps"]))
    assert np.abs(rms - fx["rms"]).max() <= 2e-6 * np.abs(fx["rms"]).max()
    sw = oracle.silu_mul(fx["gate"], fx["up"])
    assert np.abs(sw - fx["swiglu"]).max() <= 2e-6 * np.abs(fx["swiglu"]).max()
    # RoPE table (generate.zig:791-808) vs the tool's float32 inv_freq/cos/sin.
    # Angles reach ~8 rad, so allow a few ulp of the angle.
    cos, sin = oracle.rope_table(fx["rope_cos"].shape[0], int(fx["table_dim"]), float(fx["theta"]))
    assert np.abs(cos - fx["rope_cos"]).max() < 4e-6
    assert np.abs(sin - fx["rope_sin"]).max() < 4e-6
    # Softmax order of the attention kernel (max, exp, sum, scale) vs reference softmax:
    s = fx["scores"].astype(np.float32)
    e = np.exp(s - s.max(axis=1, keepdims=True))
    assert np.abs(e / e.sum(axis=1, keepdims=True) - fx["probs"]).max() < 1e-6


def test_rope_known_answers():
    # forward.zig:1265-1288: position 0 identity; position 1 rotates pair 0 by 1 rad.
    cos, sin = oracle.rope_table(2, 4, 10000.0)
    row = np.array([3, 7, -2, 5], np.float32)
    assert oracle.rope_apply(cos, sin, row, 0, 1, 4).tolist() == row.tolist()
    got = oracle.rope_apply(cos, sin, np.array([1, 0, 0, 0], np.float32), 1, 1, 4)
    assert abs(got[0] - math.cos(1.0)) < 1e-5 and abs(got[2] - math.sin(1.0)) < 1e-5


def test_add_rmsnorm_matches_add_then_norm():
    # kernels.zig:322 fused residual == addInto + rmsNormF32 byte for byte
    rng = np.random.default_rng(5)
    a = rng.standard_normal((3, 200), dtype=np.float32)
    b = rng.standard_normal((3, 200), dtype=np.float32)
    w = rng.standard_normal(200, dtype=np.float32)
    res, out = oracle.add_rmsnorm(a, b, w, 1e-6)
    assert res.tobytes() == (a + b).tobytes()
    assert out.tobytes() == oracle.rmsnorm(a + b, w, 1e-6).tobytes()


# --- sampling.zig tests ------------------------------------------------------------------

def test_eligible_argmax_mask_geometry():
    # sampling.zig:223-250
    lg = np.zeros(65, np.float32)
    for words in ([], [1], [1, 0, 0], [0, 0], [1, 0b10]):
        with pytest.raises(oracle.EligibleArgmaxError, match="InvalidEligibleMask"):
            oracle.argmax_eligible(lg, words)
    with pytest.raises(oracle.EligibleArgmaxError, match="InvalidEligibleMask"):
        oracle.argmax_eligible(np.zeros(0, np.float32), [])


def test_eligible_argmax_scans_set_bits_only():
    # sampling.zig:252-263
    lg = np.full(130, -100, np.float32)
    lg[0], lg[5], lg[67], lg[129] = np.nan, 3.0, 9.0, 8.0
    assert oracle.argmax_eligible(lg, [1 << 5, 1 << 3, 1 << 1]) == (67, 3)


def test_eligible_argmax_rejects_eligible_nan_and_ties_lowest():
    # sampling.zig:265-286
    with pytest.raises(oracle.EligibleArgmaxError, match="NaN"):
        oracle.argmax_eligible(np.array([10, np.nan, 20], np.float32), [0b110])
    inf = np.float32(np.inf)
    assert oracle.argmax_eligible(np.array([0, inf, 7, inf], np.float32), [0b1010])[0] == 1
    assert oracle.argmax_eligible(np.array([0, -inf, 7, -inf], np.float32), [0b1010])[0] == 1
    assert oracle.argmax_eligible(np.array([5, 0, 5, 0], np.float32), [0b0101])[0] == 0


def test_plain_argmax_first_max_wins():
    # sampling.zig:115 greedy and :194 argmax (strict >)
    assert oracle.argmax(np.array([1, 5, 2, 4], np.float32)) == 1
    assert oracle.argmax(np.array([2, 7, 7, 1], np.float32)) == 1


# --- paged attention -----------------------------------------------------------------------

def _attention64(q, K, V, heads, kv_heads, hd):
    out = np.zeros(heads * hd)
    g = heads // kv_heads
    for h in range(heads):
        kh = K[:, (h // g) * hd:(h // g + 1) * hd].astype(np.float64)
        s = kh @ q[h * hd:(h + 1) * hd].astype(np.float64) / math.sqrt(hd)
        p = np.exp(s - s.max())
        out[h * hd:(h + 1) * hd] = (p / p.sum()) @ V[:, (h // g) * hd:(h // g + 1) * hd]
    return out


def test_paged_attention_page_placement_is_byte_identical():
    # paged_attention.zig:317-399: paged == contiguous, across page boundaries.
    rng = np.random.default_rng(11)
    L, heads, kvh, hd, seq = 2, 4, 2, 16, 37
    kvd = kvh * hd
    pf = oracle.page_floats(L, kvd)
    npages = -(-seq // 16)
    K = rng.standard_normal((L, seq, kvd), dtype=np.float32)
    V = rng.standard_normal((L, seq, kvd), dtype=np.float32)
    q = rng.standard_normal(heads * hd, dtype=np.float32)
    outs = []
    for bt in (np.arange(npages), np.array([5, 0, 3])):
        pool = np.zeros(pf * 6, np.float32)
        for layer in range(L):
            for p in range(seq):
                oracle.kv_append(pool, pf, bt, p, layer, kvd, K[layer, p], V[layer, p])
        outs.append(oracle.paged_attention(q, pool, pf, bt, seq, 1, heads, kvh, hd))
    assert outs[0].tobytes() == outs[1].tobytes()
    ref = _attention64(q, K[1], V[1], heads, kvh, hd)
    assert np.abs(outs[0] - ref).max() < 1e-5


def test_page_payload_offset_geometry():
    # paged_kv_cache.zig:1421-1442
    assert oracle.page_payload_offset(0, False, 0, 128) == 0
    assert oracle.page_payload_offset(0, True, 0, 128) == 16 * 128
    assert oracle.page_payload_offset(3, True, 5, 64) == ((3 * 2 + 1) * 16 + 5) * 64
