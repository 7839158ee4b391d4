"""The `.glrt` prepared runtime-image reader in the library (host code, no GPU).

Restates the reference's runtime-image, loader-schema and layout tests
(src/model/runtime_image.zig:1810-2193, src/loader.zig:1826-2990,
src/int4_weights.zig:476-840): round trips of every encoding and layout,
each corruption and descriptor rejection with its error, the independence
of CRC and digest checks, the prepared-model schema, and the rows4_k16 /
rows4 scale / PairNibble known answers.  Images come from tests/glrt_writer.py.
"""
import struct

import numpy as np
import pytest

import glrt_writer as gr
from glacier_b200 import _lib
from glacier_b200.glacier_file import reason_name
from glacier_b200.runtime_image import (RuntimeImage, pair_nibble_split, rows4_k16_to_row_major,
                                        rows4_scales_to_row_major)

CFG = dict(dim=64, hidden=128, layers=1, vocab=32, heads=4, head_dim=16, kv_heads=2, eps=1e-6, theta=1e6, tie=False)


def small_model(group=16, seed=0):
    from glacier_b200.model import ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=1, dim=64, hidden=128, num_heads=4, num_kv_heads=2, head_dim=16, vocab=32,
                      group=group)
    m = SyntheticModel(cfg, seed=seed)
    rng = np.random.default_rng(seed + 1)
    emb = (rng.integers(0, 256, cfg.vocab * cfg.dim // 2, dtype=np.uint8),
           (rng.integers(1, 16, cfg.vocab * cfg.dim // group) * 2.0 ** -8).astype(np.float32))
    return m, emb


def image(version=2, policy="portable", **kw):
    m, emb = small_model()
    return gr.build(gr.model_records(m, emb, **kw), gr.model_cfg(m), version=version, policy=policy)


def reason(fn):
    with pytest.raises(_lib.GlacierCudaError) as e:
        fn()
    assert e.value.code == _lib.EFORMAT, e.value
    return reason_name(e.value)


def open_reason(img, **kw):
    return reason(lambda: RuntimeImage(bytes(img), **kw))


@pytest.mark.parametrize("kw", [dict(), dict(layout="rows4_k16", scale_streams=("rows4",)),
                                dict(layout="rows4_k16", scale_streams=("f32", "f16", "rows4")),
                                dict(scale_streams=("f16",)), dict(mlp="pair")])
def test_round_trip_records_and_schema(kw):
    img = image(**kw)
    r = RuntimeImage(bytes(img))
    assert r.info.version == 2 and r.info.abi_policy == 1 and r.info.dim == 64 and r.info.num_kv_heads == 2
    recs = r.records()
    assert len(recs) == r.num_records == (12 if kw.get("mlp") == "pair" else 13) + 2
    mi = r.model_info()
    assert mi.mlp_layout == (2 if kw.get("mlp") == "pair" else 1) and mi.group_size == 16
    for e in recs:
        for s in range(5):
            assert (e.stream_offset[s] == 0) == (e.stream_len[s] == 0)
            assert e.stream_offset[s] % 64 == 0


def test_v1_images_and_policies():
    img = image(version=1)
    r = RuntimeImage(bytes(img))
    assert r.info.version == 1 and r.model_info().mlp_layout == 1
    assert open_reason(img, allow_v1=False) == "LegacyVersionDisabled"
    a = image(policy="aarch64")
    assert RuntimeImage(bytes(a)).info.abi_policy == 2
    assert open_reason(a, abi_policy="portable") == "AbiFingerprintMismatch"
    assert open_reason(image(), abi_policy="aarch64") == "AbiFingerprintMismatch"
    # PairNibble is undefined in v1 (runtime_image.zig:444).
    m, emb = small_model()
    v1pair = gr.build(gr.model_records(m, emb, mlp="pair"), gr.model_cfg(m), version=1)
    assert open_reason(v1pair) in ("BadRole", "BadVersionedRecord", "BadEncoding")


def test_payload_crc_and_digest_are_independent():
    """runtime_image.zig:1968-2083 and loader.zig:2951: corruption, digest binding, skip options."""
    img = image()
    r = RuntimeImage(bytes(img))
    e = r.record(5)
    bad = bytearray(img)
    bad[e.stream_offset[0]] ^= 0x40
    assert open_reason(bad) == "CrcMismatch"
    assert open_reason(bad, verify_crc=False) == "DigestMismatch"
    assert open_reason(bad, verify_digest=False) == "CrcMismatch"
    RuntimeImage(bytes(bad), verify_crc=False, verify_digest=False)
    # A changed stored digest (index and header CRCs refreshed) fails only the digest check.
    d = bytearray(img)
    d[512 + 5 * 160 + 140] ^= 1
    gr.refresh_crcs(d)
    assert open_reason(d) == "DigestMismatch"
    RuntimeImage(bytes(d), verify_digest=False)
    # The digest binds the descriptor: a payload CRC field edited to match nothing fails the
    # CRC check, and with CRC checks off the digest over bytes 0..128 still catches it.
    g = edit(img, 512 + 5 * 160 + 28, "<I", 0x12345678)
    assert open_reason(g) == "CrcMismatch"
    assert open_reason(g, verify_crc=False) == "DigestMismatch"
    assert open_reason(img, expected_source_fingerprint=b"\x22" * 32) == "SourceFingerprintMismatch"
    RuntimeImage(bytes(img), expected_source_fingerprint=b"\x11" * 32)


def edit(img, off, fmt, value, refresh=True):
    b = bytearray(img)
    struct.pack_into(fmt, b, off, value)
    if refresh:
        gr.refresh_crcs(b)
    return b


REC0 = 512  # first record


@pytest.mark.parametrize("off,fmt,value,refresh,want", [
    (0, "<4s", b"GLRX", True, "BadMagic"),
    (4, "<H", 3, True, "BadVersion"),
    (6, "<H", 256, True, "BadHeaderSize"),
    (8, "<H", 128, True, "BadRecordSize"),
    (10, "<H", 32, True, "BadAlignment"),
    (140, "<B", 2, True, "BadConfig"),
    (141, "<B", 1, True, "BadReservedField"),
    (300, "<B", 1, True, "BadReservedField"),
    (144, "<f", 0.0, True, "BadConfig"),
    (148, "<f", float("inf"), True, "BadConfig"),
    (112, "<I", 0, True, "BadConfig"),
    (100, "<B", 7, False, "HeaderCrcMismatch"),
    (12, "<I", 1, True, "BadHeader"),
    (16, "<Q", 0, True, "BadHeader"),
    (40, "<Q", 1 << 40, True, "BadBounds"),
    (24, "<Q", 576, True, "BadBounds"),
    (32, "<Q", 520, True, "BadAlignment"),
    (REC0 + 16, "<I", 5, False, "IndexCrcMismatch"),
    (REC0 + 24, "<I", 1, True, "BadFlags"),
    (REC0 + 124, "<I", 1, True, "BadReservedField"),
    (REC0 + 4, "<I", 16, True, "BadTensorKind"),
    (REC0 + 8, "<H", 3, True, "BadEncoding"),
    (REC0 + 10, "<H", 2, True, "BadPackedLayout"),
    (REC0 + 120, "<H", 2, True, "BadRole"),
    (REC0 + 122, "<H", 1, True, "BadPairNibbleLayout"),
    (REC0 + 128, "<32s", b"\0" * 32, True, "MissingDigest"),
    (REC0 + 20, "<I", 63, True, "BadTensorShape"),
    (REC0 + 12, "<I", 4, True, "BadEncoding"),        # raw record with a group
    (REC0 + 104, "<Q", 600, True, "BadAlignment"),    # raw stream before data_offset
])
def test_header_and_descriptor_rejections(off, fmt, value, refresh, want):
    assert open_reason(edit(image(), off, fmt, value, refresh)) == want


def test_bounds_overlap_duplicate_and_scales():
    img = image()
    r = RuntimeImage(bytes(img))
    # Record 5 is an INT4 projection: packed + f32 scales.
    base = REC0 + 5 * 160
    e = r.record(5)
    assert e.encoding == 1
    # Offset not 64-aligned; stream past the end; streams of one record overlapping.
    assert open_reason(edit(img, base + 56, "<Q", e.stream_offset[1] + 4)) == "BadAlignment"
    assert open_reason(edit(img, base + 56, "<Q", (len(img) // 64) * 64)) == "BadBounds"
    assert open_reason(edit(img, base + 56, "<Q", e.stream_offset[0])) == "OverlappingPayload"
    # An offset without a length.
    assert open_reason(edit(img, base + 72, "<Q", e.stream_offset[1])) == "BadBounds"
    # A stream overlapping an earlier record's stream.
    e4 = r.record(4)
    assert open_reason(edit(img, base + 56, "<Q", e4.stream_offset[4] if e4.stream_len[4] else
                            e4.stream_offset[0])) == "OverlappingPayload"
    # No scale stream at all; wrong packed length.
    b = edit(img, base + 56, "<Q", 0, refresh=False)
    b = edit(b, base + 64, "<Q", 0)
    assert open_reason(b) == "MissingScales"
    assert open_reason(edit(img, base + 48, "<Q", e.stream_len[0] - 1)) == "BadTensorShape"
    # A duplicate (layer, kind) identity: record 6 repeats record 5's and fails before its own
    # digest is checked; the same edit on record 5 fails record 5's digest first (index order).
    assert open_reason(edit(img, base + 160 + 4, "<I", e.tensor_kind)) == "DuplicateRecord"
    assert open_reason(edit(img, base + 4, "<I", r.record(6).tensor_kind)) == "DigestMismatch"


def test_rows4_layout_needs_rows4_geometry():
    m, emb = small_model()
    recs = gr.model_records(m, emb, layout="rows4_k16", scale_streams=("f32",))  # no rows4 scale grid
    assert open_reason(gr.build(recs, gr.model_cfg(m))) == "BadPackedLayout"


def schema_reason(recs, cfg):
    img = RuntimeImage(bytes(gr.build(recs, cfg)))
    return reason(img.model_info)


def test_prepared_schema_rejections():
    """loader.zig:1826 (extra layer / global tensors), :2583 (pair coexistence, partial branches, mixed layers)."""
    m, emb = small_model()
    cfg = gr.model_cfg(m)
    recs = gr.model_records(m, emb)
    extra = recs + [gr.raw_rec(1, "input_norm", m.layers[0]["input_norm"])]
    assert schema_reason(extra, cfg) == "BadPayload"
    assert schema_reason(recs + [gr.raw_rec(gr.GLOBAL, "attn_q_bias", np.zeros(64))], cfg) == "BadPayload"
    tied = dict(cfg, tie=True)
    assert schema_reason(recs, tied) == "BadPayload"  # an lm_head record in a tied model
    no_up = [r for r in recs if not (r.layer == 0 and r.kind == 5)]
    assert schema_reason(no_up, cfg) == "MissingTensor"
    both = recs + [gr.pair_rec(0, m.layers[0]["wg"], m.layers[0]["wu"], 128, 64, 16)]
    assert schema_reason(both, cfg) == "BadPayload"
    bad_heads = dict(cfg, heads=3)
    assert schema_reason(recs, bad_heads) == "BadPayload"
    # Two layers, one PairNibble and one separate: the MLP form must be homogeneous.
    from glacier_b200.model import ModelConfig, SyntheticModel
    m2 = SyntheticModel(ModelConfig(num_layers=2, dim=64, hidden=128, num_heads=4, num_kv_heads=2, head_dim=16,
                                    vocab=32, group=16), seed=3)
    sep = gr.model_records(m2, emb)
    pr = gr.model_records(m2, emb, mlp="pair")
    mixed = [r for r in sep if r.layer != 1] + [r for r in pr if r.layer == 1]
    assert schema_reason(mixed, gr.model_cfg(m2)) == "BadPayload"
    # A wrong gate shape surfaces from preparedInt4 inside the record-set check.
    wrong = [r for r in recs if not (r.layer == 0 and r.kind == 7)]
    wrong.append(gr.int4_rec(0, "mlp_gate", *m.layers[0]["wd"], 64, 128, 16))
    assert schema_reason(wrong, cfg) == "BadPayload"


def test_rows4_k16_known_answer():
    """int4_weights.zig:492-523: nibble row*4 + col%4 over 4 x 32 packs to 0x10 0x32 ... 0xfe."""
    out_f, in_f = 4, 32
    logical = np.array([[r * 4 + c % 4 for c in range(in_f)] for r in range(out_f)], np.uint8).reshape(-1)
    tiled = gr.to_rows4(gr.pack(logical), out_f, in_f)
    assert tiled[:8].tolist() == [0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE]
    assert np.array_equal(rows4_k16_to_row_major(tiled, out_f, in_f), gr.pack(logical))
    rng = np.random.default_rng(0)
    pk = rng.integers(0, 256, 8 * 48 // 2, dtype=np.uint8)
    assert np.array_equal(rows4_k16_to_row_major(gr.to_rows4(pk, 8, 48), 8, 48), pk)


def test_rows4_scale_grid_known_answer():
    """int4_weights.zig:476-490: row-major scales 1..8 (4 rows, 2 groups) interleave to 1 3 5 7 2 4 6 8."""
    grid = gr.rows4_grid(np.arange(1, 9, dtype=np.float32), 4)
    assert grid.tolist() == [1, 3, 5, 7, 2, 4, 6, 8]
    assert rows4_scales_to_row_major(grid, 4, 2).tolist() == list(range(1, 9))


def test_pair_nibble_every_code_pair_and_scale_order():
    """int4_weights.zig:525-650, :790-838: all 256 gate/up pairs; scale tile/group/branch/lane order."""
    out_f, in_f, group = 16, 16, 16
    codes = np.arange(256)
    gate = gr.pack(codes & 15)
    up = gr.pack(codes >> 4)
    gs = (0x2000 + np.arange(out_f * in_f // group)).astype(np.uint16).view(np.float16).astype(np.float32)
    us = (0x6000 + np.arange(out_f * in_f // group)).astype(np.uint16).view(np.float16).astype(np.float32)
    pb, ps = gr.pair(gate, up, gs, us, out_f, in_f)
    assert sorted(pb.tolist()) == list(range(256))
    g2, u2, gs2, us2 = pair_nibble_split(pb, ps, out_f, in_f, group)
    assert np.array_equal(g2, gate) and np.array_equal(u2, up)
    assert np.array_equal(gs2, gs) and np.array_equal(us2, us)
    # Asymmetric g8 shape: 8 x 16, two groups per row.
    rng = np.random.default_rng(9)
    ga, ua = rng.integers(0, 256, 64, dtype=np.uint8), rng.integers(0, 256, 64, dtype=np.uint8)
    gsa = (0x2100 + np.arange(16)).astype(np.uint16).view(np.float16).astype(np.float32)
    usa = (0x6100 + np.arange(16)).astype(np.uint16).view(np.float16).astype(np.float32)
    pb, ps = gr.pair(ga, ua, gsa, usa, 8, 16)
    psb = ps.view(np.uint16)
    assert psb[:8].tolist() == [0x2100, 0x2102, 0x2104, 0x2106, 0x6100, 0x6102, 0x6104, 0x6106]
    g2, u2, gs2, us2 = pair_nibble_split(pb, ps, 8, 16, 8)
    assert np.array_equal(g2, ga) and np.array_equal(u2, ua) and np.array_equal(gs2, gsa)
    assert np.array_equal(us2, usa)


def test_large_image_parallel_verification():
    """Over 32 MiB of streams takes the multi-threaded CRC/digest path; the first bad record is reported."""
    recs = [gr.raw_rec(0, "other", np.full(1 << 18, i, np.float32)) for i in range(40)]
    for i, r in enumerate(recs):
        r.layer = i  # distinct identities
    img = gr.build(recs, CFG)
    r = RuntimeImage(bytes(img))
    bad = bytearray(img)
    for i in (31, 7):
        bad[r.record(i).stream_offset[4] + 100] ^= 1
    with pytest.raises(_lib.GlacierCudaError) as e:
        RuntimeImage(bytes(bad))
    assert reason_name(e.value) == "CrcMismatch" and "record 7:" in str(e.value)
    with pytest.raises(_lib.GlacierCudaError) as e:
        RuntimeImage(bytes(bad), verify_crc=False)
    assert reason_name(e.value) == "DigestMismatch" and "record 7:" in str(e.value)


def test_open_from_path(tmp_path):
    path = tmp_path / "m.glrt"
    path.write_bytes(bytes(image()))
    r = RuntimeImage(str(path))
    assert r.num_records == 15 and r.model_info().group_size == 16


def test_bulk_record_query_matches_single_queries():
    r = RuntimeImage(bytes(image(mlp="pair")))
    bulk = r.records()
    assert len(bulk) == r.num_records
    for i, e in enumerate(bulk):
        one = r.record(i)
        assert (e.layer_idx, e.tensor_kind, e.role, bytes(e.payload_digest)) == \
            (one.layer_idx, one.tensor_kind, one.role, bytes(one.payload_digest))


@pytest.mark.parametrize("kw", [dict(), dict(layout="rows4_k16", scale_streams=("rows4",)), dict(mlp="pair"),
                                dict(scale_streams=("f16",), tie=True)])
def test_host_model_reassembles_the_prepared_model(kw):
    """Every prepared layout comes back as the row-major tensors it was prepared from, so
    tensor-parallel shards cut from the image equal the shards cut from the model."""
    from glacier_b200.model import TensorParallelShard
    from glacier_b200.runtime_image import host_model
    kw = dict(kw)
    tie = kw.pop("tie", False)
    m, emb = small_model()
    hm = host_model(bytes(gr.build(gr.model_records(m, emb, tie=tie, **kw), gr.model_cfg(m, tie=tie))))
    assert {k: hm.cfg[k] for k in ("num_layers", "dim", "hidden", "num_heads", "num_kv_heads", "head_dim", "vocab",
                                   "group")} == {k: m.cfg[k] for k in ("num_layers", "dim", "hidden", "num_heads",
                                                                       "num_kv_heads", "head_dim", "vocab", "group")}
    for La, Lb in zip(hm.layers, m.layers):
        for k, v in Lb.items():
            if isinstance(v, tuple):
                assert all(np.array_equal(x, y) for x, y in zip(La[k], v)), k
            else:
                assert np.array_equal(La[k], v), k
    q = np.stack([emb[0] & 15, emb[0] >> 4], -1).reshape(-1).astype(np.float32) - 7
    assert np.array_equal(hm.embedding.ravel(), q * np.repeat(emb[1], 16))
    head = emb if tie else m.lm_head
    assert np.array_equal(hm.lm_head[0], head[0]) and np.array_equal(hm.lm_head[1], head[1])
    sa, sb = TensorParallelShard(hm, 0, 2), TensorParallelShard(m, 0, 2)
    for La, Lb in zip(sa.layers, sb.layers):
        for k, v in Lb.items():
            if isinstance(v, tuple):
                assert all(np.array_equal(x, y) for x, y in zip(La[k], v)), k


@pytest.mark.parametrize("drop", [("layer", "mlp_down"), ("global", "final_norm"), ("global", "embedding"),
                                  ("global", "lm_head")])
def test_host_model_rejects_an_incomplete_image(drop):
    """An image missing a tensor the decode path needs ends in a ValueError naming the gap
    (from the reader's schema check or from HostModel), never in a later TypeError or KeyError."""
    from glacier_b200.runtime_image import host_model
    m, emb = small_model()
    recs = gr.model_records(m, emb)
    want = gr.gw.KIND[drop[1]]
    keep = [r for r in recs if not (r.kind == want and ((r.layer == gr.GLOBAL) == (drop[0] == "global"))
                                    and (drop[0] == "global" or r.layer == 0))]
    assert len(keep) == len(recs) - 1
    with pytest.raises(ValueError):
        host_model(bytes(gr.build(keep, gr.model_cfg(m))))
