"""Kernels (c), (d), (e) on the GPU vs the CPU oracle."""
import math

import numpy as np
import pytest

import oracle
from helpers import REL_TOL, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("dim", [896, 3584, 200, 18944])
def test_rmsnorm_and_fused_residual(dim):
    from glacier_b200 import ops
    rng = np.random.default_rng(dim)
    a = rng.standard_normal((3, dim), dtype=np.float32) * 3
    b = rng.standard_normal((3, dim), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    got = host(ops.rms_norm_f32(dev(a), dev(w), 1e-6))
    assert max_rel_err(got, oracle.rmsnorm(a, w, 1e-6)) <= 1e-5
    res, out = ops.add_rms_norm_f32(dev(a), dev(b), dev(w), 1e-6)
    ref_res, ref_out = oracle.add_rmsnorm(a, b, w, 1e-6)
    assert host(res).tobytes() == ref_res.tobytes()  # the add itself is exact
    assert max_rel_err(host(out), ref_out) <= 1e-5


def test_silu_mul_rows():
    from glacier_b200 import ops
    rng = np.random.default_rng(1)
    gu = rng.standard_normal((4, 2 * 4864), dtype=np.float32) * 4
    g, u = gu[:, :4864], gu[:, 4864:]
    t = dev(gu)
    got = host(ops.silu_mul_f32(t[:, :4864], t[:, 4864:]))
    ref = np.stack([oracle.silu_mul(g[i], u[i]) for i in range(4)])
    assert max_rel_err(got, ref) <= 1e-5


def test_embedding_gather_and_bad_token():
    from glacier_b200 import ops, _lib
    rng = np.random.default_rng(2)
    table = rng.standard_normal((1000, 64)).astype(np.float16)
    toks = np.array([0, 999, 17], np.int32)
    got = host(ops.load_embedding_rows(dev(table).view(torch.int16), dev(toks)))
    assert got.tobytes() == table[toks].astype(np.float32).tobytes()
    _lib.lib().glacier_cuda_device_status(1)


@pytest.mark.parametrize("heads,kv_heads,hd", [(28, 4, 128), (14, 2, 64), (12, 2, 128)])
def test_qkv_rope_append_matches_oracle(heads, kv_heads, hd):
    from glacier_b200 import ops
    rng = np.random.default_rng(heads)
    L, layer, lanes, max_pages = 3, 1, 2, 4
    qd, kvd = heads * hd, kv_heads * hd
    pf = oracle.page_floats(L, kvd)
    cos, sin = oracle.rope_table(64, hd, 1e6)
    qkv = rng.standard_normal((lanes, qd + 2 * kvd), dtype=np.float32)
    bias = rng.standard_normal(qd + 2 * kvd, dtype=np.float32) * 0.1
    pos = np.array([5, 37], np.int32)
    bt = np.array([[3, 1, 6, 0], [2, 7, 4, 5]], np.int32)
    pages = dev(np.zeros(8 * pf, np.float32))
    q_out = host(ops.qkv_rope_append(dev(qkv), dev(bias), dev(cos), dev(sin), dev(pos), heads, kv_heads, hd, pages,
                                     pf, dev(bt), layer))
    pool = host(pages)
    ref_pool = np.zeros(8 * pf, np.float32)
    for b in range(lanes):
        row = qkv[b] + bias
        q = oracle.rope_apply(cos, sin, row[:qd], int(pos[b]), heads, hd)
        k = oracle.rope_apply(cos, sin, row[qd:qd + kvd], int(pos[b]), kv_heads, hd)
        oracle.kv_append(ref_pool, pf, bt[b], int(pos[b]), layer, kvd, k, row[qd + kvd:])
        assert np.abs(q_out[b] - q).max() <= 1e-6 * max(1, np.abs(q).max())
    assert np.abs(pool - ref_pool).max() <= 1e-6 * max(1, np.abs(ref_pool).max())


@pytest.mark.parametrize("heads,kv_heads,hd,ctxs", [
    (28, 4, 128, [1, 17, 300, 1100]),   # 7B geometry, ragged lanes across page boundaries
    (14, 2, 64, [512, 513]),            # 0.5B geometry
    (12, 2, 128, [2048]),
    (4, 4, 64, [33]),                   # no GQA sharing
    # 8 lanes of the 7B geometry at long contexts: the most segment slots the combine's
    # shared-memory weight table holds (the strong-scaling share of one GPU out of 8)
    (28, 4, 128, [4000, 3000, 100, 4096, 2500, 17, 1200, 3999]),
])
def test_paged_attention_matches_oracle(heads, kv_heads, hd, ctxs):
    from glacier_b200 import ops
    rng = np.random.default_rng(sum(ctxs))
    L, layer = 2, 1
    kvd = kv_heads * hd
    pf = oracle.page_floats(L, kvd)
    lanes = len(ctxs)
    max_pages = max(-(-c // 16) for c in ctxs)
    # scattered page placement per lane
    perm = rng.permutation(lanes * max_pages).astype(np.int32).reshape(lanes, max_pages)
    pool = (rng.standard_normal(lanes * max_pages * pf, dtype=np.float32))
    q = rng.standard_normal((lanes, heads * hd), dtype=np.float32)
    out = host(ops.paged_attention_f32(dev(q), dev(pool), pf, dev(perm), dev(np.array(ctxs, np.int32)),
                                       max_pages * 16, layer, heads, kv_heads, hd))
    for b, c in enumerate(ctxs):
        ref = oracle.paged_attention(q[b], pool, pf, perm[b], c, layer, heads, kv_heads, hd)
        assert max_rel_err(out[b], ref) <= REL_TOL, b


def test_paged_attention_clamps_a_context_past_the_block_table():
    """A context longer than the block table covers (here 70 positions over 4 pages) is
    clamped to the table's 64 positions: the kernels never index past the lane's table row,
    and the lane attends exactly what the table holds."""
    from glacier_b200 import ops
    rng = np.random.default_rng(5)
    heads, kv_heads, hd, layer, L = 8, 2, 64, 0, 1
    pf = oracle.page_floats(L, kv_heads * hd)
    max_pages = 4
    bt = np.arange(2 * max_pages, dtype=np.int32).reshape(2, max_pages)
    pool = rng.standard_normal(2 * max_pages * pf, dtype=np.float32)
    q = rng.standard_normal((2, heads * hd), dtype=np.float32)
    out = host(ops.paged_attention_f32(dev(q), dev(pool), pf, dev(bt), dev(np.array([40, 70], np.int32)),
                                       max_pages * 16, layer, heads, kv_heads, hd))
    for b, c in enumerate([40, 64]):
        ref = oracle.paged_attention(q[b], pool, pf, bt[b], c, layer, heads, kv_heads, hd)
        assert max_rel_err(out[b], ref) <= REL_TOL, b


def test_argmax_eligible_semantics():
    from glacier_b200 import ops
    # sampling.zig:252-286 cases, one per row, n = 130 (3 words per row).
    rows = np.full((4, 130), -100, np.float32)
    rows[0, 0], rows[0, 5], rows[0, 67], rows[0, 129] = np.nan, 3.0, 9.0, 8.0
    rows[1, :4] = [0.0, np.inf, 7.0, np.inf]
    rows[2, :4] = [5.0, 0.0, 5.0, 0.0]
    rows[3, :3] = [10.0, np.nan, 20.0]
    words = np.zeros((4, 3), np.uint64)
    words[0] = [1 << 5, 1 << 3, 1 << 1]
    words[1, 0] = 0b1010
    words[2, 0] = 0b0101
    words[3, 0] = 0b110
    toks, st = ops.argmax_eligible(dev(rows), dev(words.view(np.int64)))
    toks, st = host(toks), host(st)
    assert toks[:3].tolist() == [67, 1, 0] and st[:3].tolist() == [0, 0, 0]
    assert st[3] == -5 and toks[3] == -1  # EligibleLogitNaN
    for r in range(3):
        assert toks[r] == oracle.argmax_eligible(rows[r], words[r])[0]


def test_argmax_rejects_bad_masks():
    from glacier_b200 import ops
    lg = np.zeros((2, 65), np.float32)
    words = np.array([[0, 0], [1, 0b10]], np.uint64)  # empty mask; tail bit beyond n set
    toks, st = ops.argmax_eligible(dev(lg), dev(words.view(np.int64)))
    assert host(st).tolist() == [-4, -4]


def test_argmax_plain_large_vocab_first_max():
    from glacier_b200 import ops
    rng = np.random.default_rng(9)
    lg = rng.standard_normal((3, 152064), dtype=np.float32)
    lg[1, 100] = lg[1, 151000] = 50.0  # tie -> lowest index
    toks, st = ops.argmax_eligible(dev(lg))
    assert host(toks).tolist() == [oracle.argmax(lg[i]) for i in range(3)]
    assert host(st).tolist() == [0, 0, 0]


def test_paged_attention_64_lanes_past_the_reference_cap():
    """Config 5's attention launch: 64 lanes of the 7B geometry with lanes at contexts 4096, 4097
    and 4352 (the reference caps attention at 4096, forward.zig:386; the oracle lifts the cap)
    beside lanes drawn from [256, 4096].  Lanes share physical pages through their block tables
    (the kernel only reads them), so the pool stays small while every lane reads its own
    sequence of pages."""
    from glacier_b200 import ops
    heads, kv_heads, hd = 28, 4, 128
    rng = np.random.default_rng(4352)
    L, layer = 2, 1
    kvd = kv_heads * hd
    pf = oracle.page_floats(L, kvd)
    ctxs = rng.integers(256, 4097, size=64).astype(np.int32)
    ctxs[:3] = [4096, 4097, 4352]
    max_pages = 4352 // 16
    phys = 400
    bt = rng.integers(0, phys, size=(64, max_pages)).astype(np.int32)
    pool = rng.standard_normal(phys * pf, dtype=np.float32)
    q = rng.standard_normal((64, heads * hd), dtype=np.float32)
    out = host(ops.paged_attention_f32(dev(q), dev(pool), pf, dev(bt), dev(ctxs), max_pages * 16, layer, heads,
                                       kv_heads, hd))
    for b in range(64):
        ref = oracle.paged_attention(q[b], pool, pf, bt[b], int(ctxs[b]), layer, heads, kv_heads, hd)
        assert max_rel_err(out[b], ref) <= REL_TOL, (b, int(ctxs[b]))
