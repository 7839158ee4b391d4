"""Persistent INT4 weight handles (the Metal persistent-weight API mirror), the
fused LM-head argmax and the finite check, on the GPU vs the CPU oracle.

The handle keeps f32 scales, the reference's portable numerics, so results
are compared with oracle.linear_int4 (int4_matmul.zig:215-305) at the
kernel tolerance REL_TOL; greedy ids with the oracle's argmaxEligible.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from helpers import REL_TOL, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def lib():
    from glacier_b200 import _lib
    return _lib


def p(a):
    return a.ctypes.data


@pytest.fixture
def ctx():
    L = lib()
    c = L.handle(L.lib().glacier_cuda_context_create(0))
    yield c
    L.lib().glacier_cuda_context_destroy(c)


def make(rng, out_f, in_f, group):
    n = out_f * in_f
    packed = rng.integers(0, 256, size=(n + 1) // 2, dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(-(-n // group))) * 0.02).astype(np.float32)
    return packed, scales


@pytest.mark.parametrize("out_f,in_f,group", [(4608, 3584, 32), (300, 256, 16), (37, 100, 32), (64, 96, 8),
                                              (1000, 512, 64)])
def test_dispatch_and_read_output(ctx, out_f, in_f, group):
    L = lib()
    rng = np.random.default_rng(out_f + in_f)
    packed, scales = make(rng, out_f, in_f, group)
    w = L.handle(L.lib().glacier_cuda_int4_weight_create(ctx, p(packed), packed.size, p(scales), scales.size,
                                                         group, in_f, out_f))
    try:
        x = rng.standard_normal(in_f).astype(np.float32)
        y = np.zeros(out_f, np.float32)
        L.call("glacier_cuda_int4_matvec_dispatch", ctx, w, p(x), x.size, p(y), y.size)
        assert not y.any()  # the dispatch leaves the result in the handle
        L.call("glacier_cuda_int4_weight_read_output", w, p(y), y.size)
        ref = oracle.linear_int4(x, packed, scales, out_f, in_f, group)[0]
        assert max_rel_err(y, ref) <= REL_TOL
        # Device-pointer forms: one row, then a batch of five.
        xb = rng.standard_normal((5, in_f)).astype(np.float32)
        xd = torch.from_numpy(xb).cuda()
        yd = torch.zeros((5, out_f), device="cuda")
        L.call("glacier_cuda_int4_weight_matvec", w, xd.data_ptr(), yd.data_ptr(), None, None)
        torch.cuda.synchronize()
        assert max_rel_err(yd[0].cpu().numpy(), oracle.linear_int4(xb[0], packed, scales, out_f, in_f, group)[0]) \
            <= REL_TOL
        L.call("glacier_cuda_int4_weight_matmul", w, xd.data_ptr(), in_f, yd.data_ptr(), out_f, 5, None, None)
        torch.cuda.synchronize()
        ref = oracle.linear_int4(xb, packed, scales, out_f, in_f, group)
        assert max_rel_err(yd.cpu().numpy(), ref) <= REL_TOL
        # Counts that do not cover the matrix: rejected before anything runs.
        with pytest.raises(L.GlacierCudaError):
            L.call("glacier_cuda_int4_matvec_dispatch", ctx, w, p(x), x.size - 1, p(y), y.size)
        with pytest.raises(L.GlacierCudaError):
            L.call("glacier_cuda_int4_weight_read_output", w, p(y), y.size - 1)
    finally:
        L.lib().glacier_cuda_int4_weight_destroy(w)


def test_create_rejections(ctx):
    """shim.m:4016-4025: non-power-of-two group, empty shape, short packed bytes or scales -> NULL."""
    L = lib()
    packed, scales = make(np.random.default_rng(0), 8, 64, 32)
    create = L.lib().glacier_cuda_int4_weight_create
    assert not create(ctx, p(packed), packed.size, p(scales), scales.size, 24, 64, 8)
    assert not create(ctx, p(packed), packed.size, p(scales), scales.size, 32, 0, 8)
    assert not create(ctx, p(packed), packed.size - 1, p(scales), scales.size, 32, 64, 8)
    assert not create(ctx, p(packed), packed.size, p(scales), scales.size - 1, 32, 64, 8)
    assert not create(None, p(packed), packed.size, p(scales), scales.size, 32, 64, 8)


def test_lmhead_argmax_with_masks(ctx):
    L = lib()
    rng = np.random.default_rng(7)
    vocab, dim, group, batch = 5000, 256, 32, 3
    packed, scales = make(rng, vocab, dim, group)
    w = L.handle(L.lib().glacier_cuda_int4_weight_create(ctx, p(packed), packed.size, p(scales), scales.size,
                                                         group, dim, vocab))
    try:
        x = rng.standard_normal((batch, dim)).astype(np.float32)
        words = (rng.integers(0, 2**63, size=(batch, -(-vocab // 64)), dtype=np.int64)).astype(np.int64)
        words[:, -1] &= (1 << (vocab % 64)) - 1  # no eligible bit past the vocabulary
        toks = torch.zeros(batch, dtype=torch.int32, device="cuda")
        st = torch.zeros(batch, dtype=torch.int32, device="cuda")
        logits = torch.zeros((batch, vocab), device="cuda")
        xd = torch.from_numpy(x).cuda()
        wd = torch.from_numpy(words).cuda()
        L.call("glacier_cuda_int4_weight_lmhead_argmax", w, xd.data_ptr(), batch, wd.data_ptr(), words.shape[1],
               toks.data_ptr(), st.data_ptr(), None, logits.data_ptr(), None)
        torch.cuda.synchronize()
        lg = logits.cpu().numpy()
        ref = oracle.linear_int4(x, packed, scales, vocab, dim, group)
        assert max_rel_err(lg, ref) <= REL_TOL
        assert st.cpu().tolist() == [0] * batch
        for b in range(batch):
            assert toks[b].item() == oracle.argmax_eligible(lg[b], words[b].view(np.uint64))[0]
        # Unmasked, logits kept in the handle's scratch.
        L.call("glacier_cuda_int4_weight_lmhead_argmax", w, xd.data_ptr(), batch, None, 0, toks.data_ptr(), None,
               None, None, None)
        torch.cuda.synchronize()
        for b in range(batch):
            assert toks[b].item() == oracle.argmax(lg[b])
    finally:
        L.lib().glacier_cuda_int4_weight_destroy(w)


@pytest.mark.parametrize("bad", [None, np.nan, np.inf, -np.inf])
def test_all_finite(bad):
    L = lib()
    v = np.random.default_rng(1).standard_normal(100003).astype(np.float32)
    v[-1] = np.finfo(np.float32).max
    if bad is not None:
        v[77777] = bad
    vd = torch.from_numpy(v).cuda()
    r = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    L.call("glacier_cuda_all_finite_f32", vd.data_ptr(), v.size, r.data_ptr(), None)
    assert r.item() == (1 if bad is None else 0)
    L.call("glacier_cuda_all_finite_f32", vd.data_ptr(), 0, r.data_ptr(), None)
    assert r.item() == 1


@pytest.mark.parametrize("group", [8, 16, 32])
def test_fp16_scale_handle_gemm_batches(ctx, group):
    """scale_dtype 1: the fp16 scale cache; batches above four rows run the tcgen05 GEMM."""
    L = lib()
    rng = np.random.default_rng(group)
    out_f, in_f = 2048, 1024
    packed, scales = make(rng, out_f, in_f, group)
    s16 = scales.astype(np.float16)
    w = L.handle(L.lib().glacier_cuda_int4_weight_create_ex(ctx, p(packed), packed.size, p(s16.view(np.uint16)),
                                                            s16.size, 1, group, in_f, out_f))
    try:
        ref_scales = s16.astype(np.float32)
        for batch in (1, 3, 16, 64):
            x = rng.standard_normal((batch, in_f)).astype(np.float32)
            xd = torch.from_numpy(x).cuda()
            yd = torch.zeros((batch, out_f), device="cuda")
            L.call("glacier_cuda_int4_weight_matmul", w, xd.data_ptr(), in_f, yd.data_ptr(), out_f, batch, None,
                   None)
            torch.cuda.synchronize()
            ref = oracle.linear_int4(x, packed, ref_scales, out_f, in_f, group)
            assert max_rel_err(yd.cpu().numpy(), ref) <= REL_TOL, batch
    finally:
        L.lib().glacier_cuda_int4_weight_destroy(w)
    # An unknown scale type is refused.
    assert not L.lib().glacier_cuda_int4_weight_create_ex(ctx, p(packed), packed.size, p(scales), scales.size, 2,
                                                          group, in_f, out_f)
