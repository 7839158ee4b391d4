"""Kernel (a): INT4 dequant GEMV on the GPU vs the CPU oracle (linearInt4OnTheFly)."""
import json
import os

import numpy as np
import pytest

import oracle
from helpers import REL_TOL, max_rel_err, synthetic_int4

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _run(x, packed, scales, out_f, in_f, group, bias=None):
    from glacier_b200 import ops
    y = ops.linear_int4_on_the_fly(_dev(x), _dev(packed), _dev(scales), out_f, in_f, group,
                                   bias=None if bias is None else _dev(bias))
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("out_f,in_f,group,batch", [
    (4864, 896, 32, 1),    # BASELINE config 1 (scale rows of 56 B -> FFMA2 kernel)
    (4608, 3584, 32, 1),   # 7B fused QKV (tensor-core GEMV, cluster K-split)
    (1000, 2048, 32, 3),   # row tail + K-split + batch 3
    (37888, 3584, 32, 4),  # 7B gate+up, four activation rows
    (256, 256, 32, 2),
    (4864, 896, 32, 2),
    (4864, 896, 32, 3),
    (896, 4864, 32, 1),    # down projection shape
    (3584, 18944, 32, 1),  # 7B down projection
    (1000, 256, 16, 1),
    (1000, 256, 8, 2),
    (512, 512, 64, 1),
    (300, 1024, 128, 1),
    (37, 64, 8, 1),        # tests/metal_correctness.zig:328 shape
    (5, 20, 12, 1),        # groups cross rows -> generic kernel
    (7, 40, 8, 2),         # K not a multiple of 32 -> generic kernel
])
@pytest.mark.parametrize("scale_dtype", ["f16", "f32"])
def test_gemv_matches_oracle(out_f, in_f, group, batch, scale_dtype):
    rng = np.random.default_rng(out_f * 7 + in_f + group)
    packed, s32, s16 = synthetic_int4(rng, out_f, in_f, group)
    x = rng.standard_normal((batch, in_f), dtype=np.float32)
    bias = rng.standard_normal(out_f, dtype=np.float32) * 0.1
    ref = oracle.linear_int4(x, packed, s32, out_f, in_f, group, bias=bias)
    y = _run(x, packed, s16 if scale_dtype == "f16" else s32, out_f, in_f, group, bias)
    assert max_rel_err(y, ref) <= REL_TOL


def test_formula_fixture_g8_and_g32():
    fx_all = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "int4_formula.json")))
    for key in ("4864x896_g8", "4864x896_g32", "37x64_g8"):
        fx = fx_all[key]
        i = np.arange(fx["out_f"] * fx["in_f"], dtype=np.int64)
        w = (((i * 29 + 7) % 101).astype(np.float32) - np.float32(50)) / np.float32(127)
        j = np.arange(fx["in_f"], dtype=np.int64)
        x = (((j * 13 + 3) % 47).astype(np.float32) - np.float32(23)) / np.float32(31)
        packed, scales = oracle.quantize(w, fx["group"])
        y = _run(x[None], packed, scales, fx["out_f"], fx["in_f"], fx["group"])[0]
        ref = np.array(fx["y"], np.float32)
        assert max_rel_err(y, ref) <= REL_TOL
        # tests/metal_correctness.zig:328-380 bound for the GPU matvec: 2e-5 abs.
        if key == "37x64_g8":
            assert np.abs(y - ref).max() <= 2e-5


def test_gemv_rejects_zero_group_without_writing():
    from glacier_b200 import GlacierCudaError, ops
    x = torch.zeros(64, device="cuda")
    out = torch.full((1, 8), 3.0, device="cuda")
    with pytest.raises(GlacierCudaError):
        ops.linear_int4_on_the_fly(x, torch.zeros(256, dtype=torch.uint8, device="cuda"),
                                   torch.zeros(16, device="cuda"), 8, 64, 0, out=out)
    assert (out == 3.0).all()


def test_device_status_clean_after_gemv():
    from glacier_b200 import _lib
    assert _lib.lib().glacier_cuda_device_status(1) == 0


# ---------------------------------------------------------------------------
# Q8-activation form (linearInt4WeightQ8 / linearInt4Q8OnTheFly): bit-identical
# ---------------------------------------------------------------------------

def _run_q8(x, packed, scales, out_f, in_f, group, bias=None):
    from glacier_b200 import _lib
    xd, pd, sd = _dev(x), _dev(packed), _dev(scales)
    bd = None if bias is None else _dev(bias)
    y = torch.empty((x.shape[0], out_f), dtype=torch.float32, device="cuda")
    _lib.call("glacier_cuda_int4_linear_q8", xd.data_ptr(), x.shape[0], pd.data_ptr(), sd.data_ptr(),
              int(scales.dtype == np.float16), None if bd is None else bd.data_ptr(), y.data_ptr(), out_f, in_f,
              group, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    from glacier_b200 import _lib as L
    assert L.lib().glacier_cuda_device_status(0) == 0
    return y.cpu().numpy()


@pytest.mark.parametrize("out_f,in_f,group,batch", [
    (512, 3584, 32, 1),     # 32-row CTAs (tensor-core Q8 path)
    (9600, 3584, 32, 1),    # 64-row CTAs
    (19200, 3584, 32, 1),   # 128-row CTAs
    (4608, 3584, 32, 3),    # 7B QKV, batch 3
    (3584, 3584, 32, 5),    # 7B O, batch 5 = 4 + 1 rows
    (1000, 256, 32, 2),     # row tail
    (4864, 896, 32, 1),     # config 1 (K % 256 != 0: generic kernel)
    (1000, 256, 16, 2),     # group 16: activation blocks of 16
    (1000, 256, 8, 1),      # group 8: activation blocks of 32 over four weight groups
    (512, 512, 64, 1),
])
@pytest.mark.parametrize("scale_dtype", ["f16", "f32"])
def test_q8_gemv_bit_identical_to_oracle(out_f, in_f, group, batch, scale_dtype):
    rng = np.random.default_rng(out_f + 3 * in_f + group)
    packed, s32, s16 = synthetic_int4(rng, out_f, in_f, group)
    x = rng.standard_normal((batch, in_f), dtype=np.float32)
    x[0, 32:64] = 0  # an all-zero activation block (scale 0)
    bias = rng.standard_normal(out_f, dtype=np.float32) * 0.1
    ref = oracle.linear_int4_q8(x, packed, s32, out_f, in_f, group, bias=bias, weight_dispatch=True)
    y = _run_q8(x, packed, s16 if scale_dtype == "f16" else s32, out_f, in_f, group, bias)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), max_rel_err(y, ref)


def test_q8_gemv_without_bias_and_reference_fallbacks():
    rng = np.random.default_rng(11)
    # no bias
    packed, s32, s16 = synthetic_int4(rng, 768, 2048, 32)
    x = rng.standard_normal((2, 2048), dtype=np.float32)
    ref = oracle.linear_int4_q8(x, packed, s32, 768, 2048, 32, weight_dispatch=True)
    assert np.array_equal(_run_q8(x, packed, s16, 768, 2048, 32).view(np.uint32), ref.view(np.uint32))
    # inputs longer than 16384 and LM-head-sized outputs take the FP32 path (oracle within tolerance)
    for out_f, in_f in ((64, 16640), (65600, 256)):
        packed, s32, s16 = synthetic_int4(rng, out_f, in_f, 32)
        x = rng.standard_normal((1, in_f), dtype=np.float32)
        ref = oracle.linear_int4_q8(x, packed, s32, out_f, in_f, 32, weight_dispatch=True)
        assert np.array_equal(ref, oracle.linear_int4(x, packed, s32, out_f, in_f, 32))
        assert max_rel_err(_run_q8(x, packed, s16, out_f, in_f, 32), ref) <= REL_TOL
