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


def test_lmhead_argmax_epilogue_matches_the_two_pass_argmax(ctx):
    """Up to four rows take the GEMV with the argmax in its epilogue; five rows take the GEMV
    then the two-pass argmax.  Both give the same records (value, index, valid, saw_nan),
    tokens and statuses, with and without a mask, and with a NaN row (scales of one output
    row set to NaN) eligible or masked out."""
    import ctypes as C
    L = lib()
    rng = np.random.default_rng(9)
    vocab, dim, group = 3000, 512, 32
    packed, scales = make(rng, vocab, dim, group)
    scales = scales.copy()
    scales.reshape(vocab, -1)[1234] = np.nan
    w = L.handle(L.lib().glacier_cuda_int4_weight_create(ctx, p(packed), packed.size, p(scales), scales.size,
                                                         group, dim, vocab))

    class Rec(C.Structure):
        _fields_ = [("value", C.c_float), ("index", C.c_size_t), ("valid", C.c_int), ("saw_nan", C.c_int)]

    try:
        x = rng.standard_normal((5, dim)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        nw = -(-vocab // 64)
        masks = {
            "none": None,
            "nan_masked_out": np.full((5, nw), -1, np.int64),
            "sparse": rng.integers(0, 2**63, size=(5, nw), dtype=np.int64),
        }
        masks["nan_masked_out"][:, 1234 // 64] &= ~(1 << (1234 % 64))
        for m in masks.values():
            if m is not None:
                m[:, -1] &= (1 << (vocab % 64)) - 1
        for name, m in masks.items():
            got = {}
            for batch in (4, 5):
                toks = torch.zeros(batch, dtype=torch.int32, device="cuda")
                st = torch.zeros(batch, dtype=torch.int32, device="cuda")
                rec = torch.zeros((batch, C.sizeof(Rec)), dtype=torch.uint8, device="cuda")
                wd = None if m is None else torch.from_numpy(m[:batch].copy()).cuda()
                L.call("glacier_cuda_int4_weight_lmhead_argmax", w, xd.data_ptr(), batch,
                       None if wd is None else wd.data_ptr(), 0 if wd is None else nw, toks.data_ptr(),
                       st.data_ptr(), rec.data_ptr(), None, None)
                torch.cuda.synchronize()
                recs = [Rec.from_buffer_copy(rec[b].cpu().numpy().tobytes()) for b in range(batch)]
                got[batch] = (toks.cpu().tolist()[:4], st.cpu().tolist()[:4],
                              [(r.value, r.index, r.valid, r.saw_nan) for r in recs[:4]])
            assert got[4] == got[5], name
            if name == "none":
                assert got[4][1] == [L.ENAN] * 4 and got[4][0] == [-1] * 4
            if name == "nan_masked_out":
                assert got[4][1] == [0] * 4
    finally:
        L.lib().glacier_cuda_int4_weight_destroy(w)


def test_fp16_scales_with_inf_and_nan_propagate(ctx):
    """A weight whose fp16 scales hold an infinity and a NaN: the NaN row comes out NaN and the
    infinity row non-finite, as in the oracle, not as the large finite numbers a finite-only
    conversion makes; every other row matches the oracle."""
    L = lib()
    rng = np.random.default_rng(11)
    M, K, G = 640, 512, 32
    packed, scales = make(rng, M, K, G)
    s16 = scales.astype(np.float16)
    s16.reshape(M, -1)[7, 3] = np.inf
    s16.reshape(M, -1)[300, 0] = np.nan
    ref_scales = s16.astype(np.float32)
    bits = s16.view(np.uint16)
    w = L.handle(L.lib().glacier_cuda_int4_weight_create_ex(ctx, p(packed), packed.size, p(bits), bits.size, 1, G,
                                                            K, M))
    try:
        x = rng.standard_normal((2, K)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        y = torch.empty((2, M), device="cuda")
        L.call("glacier_cuda_int4_weight_matmul", w, xd.data_ptr(), K, y.data_ptr(), M, 2, None, None)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        ref = oracle.linear_int4(x, packed, ref_scales, M, K, G)
        assert np.isnan(got[:, 300]).all() and np.isnan(ref[:, 300]).all()
        assert not np.isfinite(got[:, 7]).any() and not np.isfinite(ref[:, 7]).any()
        rest = np.ones(M, bool)
        rest[[7, 300]] = False
        assert np.isfinite(got[:, rest]).all() and max_rel_err(got[:, rest], ref[:, rest]) <= REL_TOL
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
