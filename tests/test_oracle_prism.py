"""The Prism progressive-INT4 scalar oracle (src/progressive_int4.zig), pinned by
the reference's own tests (tests/progressive_int4.zig:24-205): the exact
1 + 1 + 2-bit decomposition of every nibble, the little-lane plane encoding,
the plane byte lengths, and P1/P2/P4 dot products that agree bit for bit with
an independent sequential restatement and, at P4, with the legacy full-INT4
formula.  No GPU needed.
"""
import numpy as np
import pytest

import oracle

P1 = [-4] * 8 + [4] * 8
P2 = [-6] * 4 + [-2] * 4 + [2] * 4 + [6] * 4
P4 = list(range(-7, 9))


def test_decomposition_reconstructs_all_sixteen_nibbles():
    for u in range(16):
        assert oracle.prism_value(u, 1) == P1[u]
        assert oracle.prism_value(u, 2) == P2[u]
        assert oracle.prism_value(u, 4) == P4[u] == u - 7


def test_plane_split_known_answer_and_reconstruction():
    """tests/progressive_int4.zig:47-73: nibbles 0..15 -> coarse 00 ff, middle f0 f0, fine e4 x4."""
    packed = np.array([(2 * i) | ((2 * i + 1) << 4) for i in range(8)], np.uint8)
    c, m, f = oracle.prism_split(packed, 16)
    assert c.tolist() == [0x00, 0xFF] and m.tolist() == [0xF0, 0xF0] and f.tolist() == [0xE4] * 4
    for i in range(16):
        u = ((c[i // 8] >> (i % 8)) & 1) << 3 | ((m[i // 8] >> (i % 8)) & 1) << 2 | ((f[i // 4] >> (2 * (i % 4))) & 3)
        assert u == i


@pytest.mark.parametrize("n,coarse,fine", [(0, 0, 0), (1, 1, 1), (4, 1, 1), (5, 1, 2), (8, 1, 2), (9, 2, 3)])
def test_plane_byte_lengths(n, coarse, fine):
    c, m, f = oracle.prism_split(np.zeros(-(-n // 2), np.uint8), n)
    assert (c.size, m.size, f.size) == (coarse, coarse, fine)


def sequential_dot(x, values, scales, group):
    r = np.float32(0)
    for i in range(x.size):
        r = np.float32(r + np.float32(x[i] * np.float32(np.float32(values[i]) * scales[i // group])))
    return r


LENGTHS = [1, 2, 3, 5, 7, 8, 9, 15, 17, 31, 33, 63, 65, 127]
GROUPS = [1, 2, 3, 4, 5, 7, 8, 16, 31, 64, 129]


def test_p4_dot_is_the_legacy_int4_dot_at_every_tier_and_tail():
    """tests/progressive_int4.zig:105-204, with the odd-tail padding nibble set to 0xF."""
    rng = np.random.default_rng(0x676C616369657234 % 2**32)
    for n in LENGTHS:
        for g in GROUPS:
            x = (rng.random(n, dtype=np.float32) * 4 - 2).astype(np.float32)
            scales = (rng.random(-(-n // g), dtype=np.float32) * 0.5 + 0.001).astype(np.float32)
            codes = rng.integers(0, 16, n).astype(np.uint8)
            packed = np.zeros(-(-n // 2), np.uint8)
            for i, u in enumerate(codes):
                packed[i // 2] |= u << (4 * (i % 2))
            if n % 2:
                packed[-1] |= 0xF0
            dots = oracle.prism_dot_all(x, packed, scales, g)
            for t, tier in enumerate((1, 2, 4)):
                vals = [oracle.prism_value(int(u), tier) for u in codes]
                assert dots[t] == sequential_dot(x, vals, scales, g), (n, g, tier)
            assert dots[2] == sequential_dot(x, codes.astype(np.int64) - 7, scales, g)
            c, m, f = oracle.prism_split(packed, n)
            assert oracle.prism_dot_planes(x, 1, c, None, None, scales, g) == dots[0]
            assert oracle.prism_dot_planes(x, 2, c, m, None, scales, g) == dots[1]
            assert oracle.prism_dot_planes(x, 4, c, m, f, scales, g) == dots[2]
