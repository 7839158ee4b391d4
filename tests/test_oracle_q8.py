"""Pins the oracle's Q8-activation path (int4_matmul.zig:335-532) on the CPU.

* The reference's own test "q8 activation INT4 path stays close to FP32 activation
  reference" (int4_matmul.zig:3375-3423): its exact weight and input formulas, groups 8
  and 16, |Q8 - FP32 linear| <= 0.08.
* An independent numpy restatement of linearInt4Q8OnTheFly (int32 dot per group, then
  acc + (float)dot * w_scale * a_scale in float32, group by group) agrees bit for bit.
* The quantizer's rounding (half away from zero), clamping and all-zero blocks.
* The dispatch rules: inputs longer than 16384 (:369) and LM-head-sized outputs
  (out_f > 65536, :460) take the FP32 path.
No GPU needed.
"""
import numpy as np
import pytest

import oracle


def numpy_q8_quantize(x, group):
    ag = 32 if group == 8 else group
    q = np.zeros(x.size, np.int8)
    scales = np.zeros(-(-x.size // ag), np.float32)
    for g in range(scales.size):
        blk = x[g * ag:(g + 1) * ag].astype(np.float32)
        m = np.float32(np.max(np.abs(blk))) if blk.size else np.float32(0)
        scale = np.float32(m / np.float32(127.0))
        scales[g] = scale
        if scale == 0:
            continue
        inv = np.float32(np.float32(1.0) / scale)
        v = (blk * inv).astype(np.float32)
        r = np.where(v >= 0, np.floor(v.astype(np.float64) + 0.5), -np.floor(-v.astype(np.float64) + 0.5))
        q[g * ag:(g + 1) * ag] = np.clip(r, -127, 127).astype(np.int8)
    return q, scales


def numpy_linear_q8(x, packed, scales, out_f, in_f, group, bias=None):
    ag = 32 if group == 8 else group
    codes = np.stack([packed & 15, packed >> 4], -1).reshape(-1)[: out_f * in_f].astype(np.int32) - 7
    w = codes.reshape(out_f, in_f)
    out = np.zeros((x.shape[0], out_f), np.float32)
    for b in range(x.shape[0]):
        q, a_scales = numpy_q8_quantize(x[b], group)
        dots = (w.reshape(out_f, in_f // group, group) * q.astype(np.int32).reshape(in_f // group, group)).sum(-1)
        for row in range(out_f):
            acc = np.float32(bias[row]) if bias is not None else np.float32(0)
            for og in range(in_f // group):
                t = np.float32(np.float32(dots[row, og]) * np.float32(scales[(row * in_f + og * group) // group]))
                t = np.float32(t * a_scales[(og * group) // ag])
                acc = np.float32(acc + t)
            out[b, row] = acc
    return out


@pytest.mark.parametrize("group", [8, 16])
def test_reference_q8_close_to_fp32_known_case(group):
    """int4_matmul.zig:3375-3423, restated with the same source and input formulas."""
    in_f, out_f = 64, 12
    i = np.arange(in_f * out_f)
    source = (((i * 17) % 31).astype(np.float32) - 15) / np.float32(23.0)
    j = np.arange(in_f)
    inp = (((j * 7) % 19).astype(np.float32) - 9) / np.float32(11.0)
    packed, scales = oracle.quantize(source, group)
    full = oracle.dequantize(packed, scales, group, source.size).reshape(out_f, in_f)
    expected = full.astype(np.float64) @ inp.astype(np.float64)
    actual = oracle.linear_int4_q8(inp, packed, scales, out_f, in_f, group, weight_dispatch=True)[0]
    assert np.max(np.abs(actual - expected)) <= 0.08


@pytest.mark.parametrize("group,in_f,out_f,batch", [(32, 256, 24, 1), (16, 128, 17, 3), (8, 96, 9, 2),
                                                    (64, 256, 8, 1), (128, 512, 5, 2)])
def test_q8_matches_independent_numpy_restatement(group, in_f, out_f, batch):
    rng = np.random.default_rng(group * 1000 + in_f)
    packed = rng.integers(0, 256, size=out_f * in_f // 2, dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(out_f * in_f // group)) * 0.02).astype(np.float16).astype(np.float32)
    x = rng.standard_normal((batch, in_f)).astype(np.float32)
    x[0, :group] = 0  # one all-zero activation block
    bias = rng.standard_normal(out_f).astype(np.float32)
    got = oracle.linear_int4_q8(x, packed, scales, out_f, in_f, group, bias=bias)
    want = numpy_linear_q8(x, packed, scales, out_f, in_f, group, bias=bias)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q8_quantizer_rounding_clamp_and_zero_block():
    # block of 32: max 1.0 -> scale 1/127; 0.5 * 127 = 63.5 rounds away from zero to 64
    x = np.zeros(64, np.float32)
    x[0], x[1], x[2], x[3] = 1.0, -0.5, 0.5, -1.0
    q, s = oracle.q8_quantize(x, 32)
    assert s[1] == 0 and not q[32:].any()
    assert (q[:4] == [127, -64, 64, -127]).all()
    qn, sn = numpy_q8_quantize(x, 32)
    assert (q == qn).all() and np.array_equal(s, sn)
    assert oracle.lib().gor_q8_activation_group(8) == 32 and oracle.lib().gor_q8_activation_group(16) == 16


def test_q8_long_inputs_and_lm_head_take_fp32_path():
    rng = np.random.default_rng(3)
    # in_f > 16384: linearInt4Q8OnTheFly falls back to linearInt4OnTheFly (:369-371)
    in_f, out_f = 16416, 2
    packed = rng.integers(0, 256, size=out_f * in_f // 2, dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(out_f * in_f // 32)) * 0.02).astype(np.float32)
    x = rng.standard_normal(in_f).astype(np.float32)
    assert np.array_equal(oracle.linear_int4_q8(x, packed, scales, out_f, in_f, 32),
                          oracle.linear_int4(x, packed, scales, out_f, in_f, 32))
    # out_f > 65536: linearInt4WeightQ8 sends the vocabulary head to the FP32 path (:460-462)
    in_f, out_f = 32, 65540
    packed = rng.integers(0, 256, size=out_f * in_f // 2, dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(out_f * in_f // 32)) * 0.02).astype(np.float32)
    x = rng.standard_normal(in_f).astype(np.float32)
    assert np.array_equal(oracle.linear_int4_q8(x, packed, scales, out_f, in_f, 32, weight_dispatch=True),
                          oracle.linear_int4(x, packed, scales, out_f, in_f, 32))
    assert not np.array_equal(oracle.linear_int4_q8(x, packed, scales, out_f, in_f, 32),
                              oracle.linear_int4(x, packed, scales, out_f, in_f, 32))


def test_q8_rejects_groups_that_do_not_tile_the_row():
    with pytest.raises(ValueError):
        oracle.linear_int4_q8(np.zeros(40, np.float32), np.zeros(80, np.uint8), np.ones(5, np.float32), 4, 40, 32)
