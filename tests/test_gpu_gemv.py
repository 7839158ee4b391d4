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
