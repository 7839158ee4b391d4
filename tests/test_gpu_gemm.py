"""Kernel (b): tcgen05/TMEM INT4 dequant GEMM on the GPU vs the CPU oracle."""
import numpy as np
import pytest

import oracle
from helpers import REL_TOL, max_rel_err, synthetic_int4

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("out_f,in_f,batch", [
    (256, 512, 16),      # one tile, single split
    (1000, 2048, 17),    # row tail, padded batch
    (512, 1024, 5),
    (4608, 3584, 64),    # 7B fused QKV at 64 lanes
    (3584, 18944, 64),   # 7B down projection
    (256, 512, 128),     # widest batch tile
    (37888, 3584, 64),   # 7B fused gate/up at 64 lanes (the longest unit list of the persistent grid)
    (152064, 3584, 64),  # 7B LM head at 64 lanes
])
def test_gemm_matches_oracle(out_f, in_f, batch):
    from glacier_b200 import _lib, ops
    rng = np.random.default_rng(out_f + in_f + batch)
    packed, s32, s16 = synthetic_int4(rng, out_f, in_f, 32)
    x = rng.standard_normal((batch, in_f), dtype=np.float32)
    x[1] *= 1e-3   # per-row scaling of the split activation
    x[2] *= 300.0
    bias = rng.standard_normal(out_f, dtype=np.float32) * 0.1
    y = ops.linear_int4_tensor_core(dev(x), dev(packed), dev(s16.view(np.int16)), out_f, in_f, 32, bias=dev(bias))
    torch.cuda.synchronize()
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    # The oracle follows every row of the batch up to 16 and a spread of rows beyond (the
    # per-row activation scales of rows 1 and 2 among them) on the largest matrices.
    rows = np.arange(batch) if out_f * in_f * batch <= 2**33 else np.unique(np.r_[0:16, 31, 47, 63] % batch)
    ref = oracle.linear_int4(x[rows], packed, s32, out_f, in_f, 32, bias=bias, threads=16)
    y = y.cpu().numpy()
    for i, b in enumerate(rows):
        assert max_rel_err(y[b], ref[i]) <= REL_TOL, b



@pytest.mark.parametrize("group,out_f,in_f,batch", [
    (16, 1000, 2048, 17),   # two scales per 32 codes
    (8, 512, 1024, 64),     # four scales per 32 codes
    (16, 4608, 3584, 64),   # 7B QKV shape in the reference's production g16 layout
    (8, 256, 512, 128),
])
def test_gemm_groups_8_and_16_match_oracle(group, out_f, in_f, batch):
    """The tcgen05 GEMM with the reference's production group sizes (g8 / g16): the converters
    pick the scale of every 8-code word from 256/group scales per row and super-stage."""
    from glacier_b200 import _lib, ops
    rng = np.random.default_rng(out_f + in_f + batch + group)
    packed, s32, s16 = synthetic_int4(rng, out_f, in_f, group)
    x = rng.standard_normal((batch, in_f), dtype=np.float32)
    bias = rng.standard_normal(out_f, dtype=np.float32) * 0.1
    y = ops.linear_int4_tensor_core(dev(x), dev(packed), dev(s16.view(np.int16)), out_f, in_f, group, bias=dev(bias))
    torch.cuda.synchronize()
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    ref = oracle.linear_int4(x, packed, s32, out_f, in_f, group, bias=bias, threads=8)
    y = y.cpu().numpy()
    for b in range(batch):
        assert max_rel_err(y[b], ref[b]) <= REL_TOL, b