"""The `.glacier` reader in the library (host code only, no GPU).

Restates the reference's own format tests (src/model/format.zig:791-1320):
the two-page portable container, every mutation those tests make and the
error it must raise, the page-geometry and quant-sub-header rejections, the
raw-page decode known answers, and the CRC check.  Images come from
tests/glacier_writer.py (struct + zlib), a second implementation of the format.
"""
import ctypes
import json
import struct
import zlib

import numpy as np
import pytest

import glacier_writer as gw
import oracle
from glacier_b200 import _lib
from glacier_b200.glacier_file import GlacierFile, crc32, parse_sidecar, reason_name, resolve_config

# format.zig:722-732: metadata {"format":"portable-test"}, two fp16 pages of 4 elements.
TEST_META = b'{"format":"portable-test"}'
TEST_PAYLOADS = (b"abcdefgh", b"ijklmnop")
INDEX_OFF = 256 + len(TEST_META)
DATA_OFF = INDEX_OFF + 64 * 2
SIZE = DATA_OFF + 16


def portable_container() -> bytearray:
    pages = [gw.Page(i, gw.KIND["embedding"] if i == 0 else gw.KIND["other"], 4 * i, 4 * i + 4, gw.PREC["fp16"], 0,
                     p) for i, p in enumerate(TEST_PAYLOADS)]
    img = gw.build(pages, TEST_META)
    assert len(img) == SIZE
    return img


def reason_of(img) -> str:
    with pytest.raises(_lib.GlacierCudaError) as e:
        GlacierFile(bytes(img))
    assert e.value.code == _lib.EFORMAT
    return reason_name(e.value)


def put_u64(img, off, v):
    struct.pack_into("<Q", img, off, v)


def test_portable_container_admits_and_checks_crcs():
    img = portable_container()
    f = GlacierFile(bytes(img))
    assert f.num_pages == 2 and f.info.container_bytes == SIZE and f.metadata() == {"format": "portable-test"}
    p = f.pages()
    assert p[0].tensor_kind == 0 and p[1].tensor_kind == 255 and p[1].data_offset == DATA_OFF + 8
    assert p[1].crc32 == zlib.crc32(b"ijklmnop")
    f.validate_pages()
    img[DATA_OFF] = ord("X")  # format.zig:1089: one payload byte changed
    bad = GlacierFile(bytes(img))  # admission does not read payloads
    with pytest.raises(_lib.GlacierCudaError) as e:
        bad.validate_pages()
    assert reason_name(e.value) == "CrcMismatch"


@pytest.mark.parametrize("mutate,reason", [
    (lambda b: b.__setitem__(256, ord("!")), "BadMetadata"),                       # format.zig:1195
    (lambda b: put_u64(b, 8, 257), "BadLayout"),                                   # :1202
    (lambda b: put_u64(b, 24, 2**64 - 1), "IndexTooLarge"),                        # :1209
    (lambda b: put_u64(b, INDEX_OFF, 1), "BadPageId"),                             # :1216
    (lambda b: put_u64(b, INDEX_OFF + 24, 0), "BadRowRange"),                      # :1223
    (lambda b: put_u64(b, INDEX_OFF + 44, 0), "EmptyPage"),                        # :1230
    (lambda b: put_u64(b, INDEX_OFF + 64 + 36, DATA_OFF + 9), "NonContiguousPayload"),  # :1237
    (lambda b: b.extend(b"\0"), "TrailingBytes"),                                  # :1248
    (lambda b: b.__delitem__(slice(SIZE - 1, SIZE)), "TruncatedPage"),             # :1255
    (lambda b: b.__setitem__(0, ord("X")), "BadMagic"),
    (lambda b: b.__setitem__(4, 2), "BadVersion"),                                 # :1107
    (lambda b: b.__setitem__(6, 1), "BadHeaderSize"),                              # :1115
    (lambda b: b.__setitem__(48, 19), "BadPageSize"),                              # :1123
    (lambda b: b.__setitem__(52, 1), "BadReservedField"),                          # :1131
    (lambda b: b.__setitem__(255, 1), "BadReservedField"),                         # :1139
    (lambda b: struct.pack_into("<I", b, INDEX_OFF + 12, 16), "BadTensorKind"),    # :1163
    (lambda b: b.__setitem__(INDEX_OFF + 32, 255), "BadPrecision"),                # :1171
    (lambda b: b.__setitem__(INDEX_OFF + 34, 1), "BadReservedField"),              # :1178
    (lambda b: b.__setitem__(INDEX_OFF + 56, 1), "BadReservedField"),
    (lambda b: b.__setitem__(INDEX_OFF + 60, 1), "BadReservedField"),
    (lambda b: b.__delitem__(slice(200, None)), "TruncatedHeader"),
    (lambda b: put_u64(b, 16, 16 * 2**20 + 1), "MetadataTooLarge"),                # :1276
    (lambda b: put_u64(b, 24, 2**20 + 1), "IndexTooLarge"),                        # :1295
    (lambda b: put_u64(b, 16, 10**6), "BadLayout"),  # index no longer follows the metadata
])
def test_admission_rejections(mutate, reason):
    img = portable_container()
    mutate(img)
    assert reason_of(img) == reason


def test_truncated_meta_and_index():
    img = portable_container()
    # A header that promises more metadata and pages than the file holds.
    meta_len = 1000
    put_u64(img, 16, meta_len)
    put_u64(img, 32, 256 + meta_len)
    put_u64(img, 40, 256 + meta_len + 128)
    assert reason_of(img) == "TruncatedMeta"
    img = portable_container()
    put_u64(img, 24, 100)
    put_u64(img, 40, INDEX_OFF + 64 * 100)
    assert reason_of(img) == "TruncatedIndex"


def one_page(precision, group, n, payload, kind="other"):
    return gw.build([gw.Page(0, gw.KIND[kind], 0, n, gw.PREC[precision], group, payload)])


def test_page_geometry_rejections():
    """format.zig:836-876: lying precision descriptors."""
    GlacierFile(bytes(one_page("fp16", 0, 4, b"\0" * 8)))
    assert reason_of(one_page("fp16", 0, 4, b"\0" * 7)) == "BadPageGeometry"
    assert reason_of(one_page("fp16", 4, 4, b"\0" * 8)) == "BadQuantGroup"
    assert reason_of(one_page("int2", 0, 4, b"\0" * 8)) == "UnsupportedPrecision"
    assert reason_of(one_page("tri1p58", 0, 4, b"\0" * 8)) == "UnsupportedPrecision"
    n = (1 << 18) // 2 + 1
    assert reason_of(one_page("fp16", 0, n, b"\0" * (2 * n))) == "PageGeometryTooLarge"
    assert reason_of(one_page("int4", 0, 64, b"\0" * 56)) == "BadQuantGroup"
    assert reason_of(one_page("int4", 32, 65537, b"\0" * (16 + 2049 * 4 + 32769))) == "PageGeometryTooLarge"
    assert reason_of(one_page("fp32", 0, 2, b"\0" * 9)) == "BadPageGeometry"
    # 2^63 fp32 elements: the byte count overflows u64.
    img = one_page("fp32", 0, 2, b"\0" * 8)
    put_u64(img, 256 + len(b'{"format":"test"}') + 24, 2**63)
    assert reason_of(img) == "LayoutOverflow"


def test_raw_decode_known_answers():
    """format.zig:878-946: fp32 / fp16 / bf16 bytes decode to {1.0, -2.5}."""
    for prec, raw in (("fp32", bytes([0, 0, 0x80, 0x3F, 0, 0, 0x20, 0xC0])), ("fp16", bytes([0, 0x3C, 0, 0xC1])),
                      ("bf16", bytes([0x80, 0x3F, 0x20, 0xC0]))):
        f = GlacierFile(bytes(one_page(prec, 0, 2, raw)))
        assert f.decode_page(0).tolist() == [1.0, -2.5]
        out = np.empty(3, np.float32)
        with pytest.raises(_lib.GlacierCudaError) as e:
            _lib.call("glacier_cuda_glacier_page_decode_f32", f._ptr, f.size, 0, out.ctypes.data, 3)
        assert reason_name(e.value) == "SizeMismatch"


def test_fp16_decode_is_exact_for_every_bit_pattern():
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    f = GlacierFile(bytes(one_page("fp16", 0, 1 << 16, bits.tobytes())))
    got = f.decode_page(0)
    want = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_quant_payload_schema_binds_entry_geometry():
    """format.zig:948-989: an INT4 page of arange(64), group 32; sub-header byte 13 set."""
    src = np.arange(64, dtype=np.float32)
    packed, scales = oracle.quantize(src, 32)
    payload = bytearray(gw.qio_payload(64, 32, 1, scales, packed))
    f = GlacierFile(bytes(one_page("int4", 32, 64, bytes(payload))))
    f.validate_pages()
    assert np.array_equal(f.decode_page(0), oracle.dequantize(packed, scales, 32, 64))
    payload[13] = 1
    f = GlacierFile(bytes(one_page("int4", 32, 64, bytes(payload))))
    with pytest.raises(_lib.GlacierCudaError) as e:
        f.validate_pages()
    assert reason_name(e.value) == "BadQuantPayload"
    with pytest.raises(_lib.GlacierCudaError) as e:
        f.decode_page(0)
    assert reason_name(e.value) == "BadQuantPayload"
    # A sub-header that disagrees with the entry: group, element count, precision byte, magic.
    for off, val in ((8, 16), (4, 63), (12, 0), (0, 0)):
        p = bytearray(gw.qio_payload(64, 32, 1, scales, packed))
        struct.pack_into("<I" if off != 12 else "<B", p, off, val)
        f = GlacierFile(bytes(one_page("int4", 32, 64, bytes(p))))
        with pytest.raises(_lib.GlacierCudaError) as e:
            f.validate_pages()
        assert reason_name(e.value) == "BadQuantPayload", off


def test_int8_and_ragged_int4_decode():
    """core/quant.zig:114-160: (code - 127) * scale for INT8, (nibble - 7) * scale for INT4, ragged tails."""
    rng = np.random.default_rng(5)
    n, g = 77, 16
    codes = rng.integers(0, 256, n, dtype=np.uint8)
    scales = rng.random(-(-n // g), dtype=np.float32)
    f = GlacierFile(bytes(one_page("int8", g, n, gw.qio_payload(n, g, 0, scales, codes))))
    f.validate_pages()
    want = (codes.astype(np.float32) - 127) * np.repeat(scales, g)[:n]
    assert np.array_equal(f.decode_page(0), want)
    packed = rng.integers(0, 256, -(-n // 2), dtype=np.uint8)
    f = GlacierFile(bytes(one_page("int4", g, n, gw.qio_payload(n, g, 1, scales, packed))))
    nib = np.stack([packed & 15, packed >> 4], -1).reshape(-1)[:n].astype(np.float32) - 7
    assert np.array_equal(f.decode_page(0), nib * np.repeat(scales, g)[:n])


def test_decode_checks_crc_first():
    img = one_page("fp32", 0, 2, bytes(8))
    img[-1] = 1
    f = GlacierFile(bytes(img))
    with pytest.raises(_lib.GlacierCudaError) as e:
        f.decode_page(0)
    assert reason_name(e.value) == "CrcMismatch"


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 63, 1000, 1 << 20])
def test_crc32_matches_zlib(n):
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    assert crc32(data) == zlib.crc32(data)
    assert crc32(b"hello glacier") == zlib.crc32(b"hello glacier")  # format.zig:831-834


def test_parallel_crc_reports_first_bad_page():
    # Over 64 MiB of pages takes the multi-threaded path; pages 3 and 200 are corrupted.
    payload = bytes(1 << 18)
    pages = [gw.Page(0, 255, i * 65536, (i + 1) * 65536, gw.PREC["fp32"], 0, payload) for i in range(300)]
    img = gw.build(pages)
    f = GlacierFile(bytes(img))
    f.validate_pages()
    for bad in (200, 3):
        img[f.page(bad).data_offset + 5] = 1
    with pytest.raises(_lib.GlacierCudaError) as e:
        GlacierFile(bytes(img)).validate_pages()
    assert reason_name(e.value) == "CrcMismatch" and "page 3:" in str(e.value)


GOOD_JSON = ['{}', ' {"a" : [1, -2.5e+3, 0, 0.5, {"b": null}], "c": true, "d": false}\n',
             '{"s": "\\u00e9\\ud83d\\ude00\\n\\"\\/"}', '{"é": "ü✓"}', '{"a": {"a": 1}}',
             '{"x":' + '[' * 5000 + ']' * 5000 + '}']
BAD_JSON = ['', '[]', '"s"', '1', '{"a":1,}', '{"a":1}{}', '{"a":01}', '{"a":1.}', '{"a":.5}', '{"a":1e}',
            '{"a":-}', '{"a":"\x01"}', '{"a":"\\ud800"}', '{"a":"\\udc00"}', '{"a":"\\x"}', '{"a":1,"a":2}',
            '{"a":"x","\\u0061":1}', '{a:1}', "{'a':1}", '{"a":tru}', '{"a":nul}', '{"a" 1}', '{"a":[1,]}',
            '{"a":[1 2]}', '﻿{}', '{"a":1}x', '{"x":' + '[' * 5000 + '}', '{"a":+1}', '{"a":NaN}']


@pytest.mark.parametrize("meta", GOOD_JSON)
def test_metadata_json_accepted(meta):
    GlacierFile(bytes(gw.build([], meta.encode())))


@pytest.mark.parametrize("meta", BAD_JSON)
def test_metadata_json_rejected(meta):
    assert reason_of(gw.build([], meta.encode())) == "BadMetadata"


@pytest.mark.parametrize("raw", [b'{"a":"\xff"}', b'{"a":"\xc0\xaf"}', b'{"a":"\xed\xa0\x80"}',
                                 b'{"a":"\xf4\x90\x80\x80"}', b'{"a":"\xe2\x82"}'])
def test_metadata_invalid_utf8_rejected(raw):
    assert reason_of(gw.build([], raw)) == "BadMetadata"


def test_geometry_from_page_metadata_and_sidecar():
    from glacier_b200.model import ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)
    m = SyntheticModel(cfg, seed=3)
    f = GlacierFile(bytes(gw.model_image(m)))
    f.validate_pages()
    g = f.geometry()
    assert (g.num_layers, g.dim, g.hidden, g.vocab, g.group_size, g.has_lm_head, g.has_qkv_bias) == \
        (2, 256, 512, 1000, 32, 1, 1)
    # Without a sidecar: head_dim 64, dim/64 heads, as many KV heads, eps 1e-6, theta 10000 (loader.zig:1525-1541).
    c = resolve_config(g, {})
    assert (c["num_heads"], c["num_kv_heads"], c["head_dim"], c["eps"], c["theta"]) == (4, 4, 64, 1e-6, 10000.0)
    ov = parse_sidecar(json.dumps({"hidden_size": 256, "num_attention_heads": 8, "num_key_value_heads": 2,
                                   "rms_norm_eps": 1e-6, "rope_theta": 1000000, "tie_word_embeddings": False,
                                   "head_dim": "64", "vocab_size": -1, "num_layers": 2.0}))
    assert ov == {"dim": 256, "num_heads": 8, "num_kv_heads": 2, "eps": float(np.float32(1e-6)), "theta": 1e6,
                  "tie_word_embeddings": False}
    c = resolve_config(g, ov)
    assert (c["num_heads"], c["num_kv_heads"], c["head_dim"], c["theta"]) == (8, 2, 64, 1e6)
    # `a orelse b`: an invalid first key falls through to the second.
    assert parse_sidecar('{"dim": "x", "hidden_size": 64}') == {"dim": 64}


def test_empty_container_has_no_layers():
    f = GlacierFile(bytes(gw.build([])))
    assert f.num_pages == 0
    with pytest.raises(_lib.GlacierCudaError) as e:
        f.geometry()
    assert reason_name(e.value) == "NoLayers"


def test_open_from_path_is_a_read_only_mapping(tmp_path):
    """A path opens as a memory mapping of the file (nothing copied), like the reference's mmap reader."""
    path = tmp_path / "m.glacier"
    path.write_bytes(bytes(portable_container()))
    f = GlacierFile(str(path))
    assert isinstance(f._buf, np.memmap) and f.num_pages == 2
    f.validate_pages()
    (tmp_path / "empty.glacier").write_bytes(b"")
    with pytest.raises(_lib.GlacierCudaError) as e:
        GlacierFile(str(tmp_path / "empty.glacier"))
    assert reason_name(e.value) == "TruncatedHeader"


def test_bulk_page_query_matches_single_queries():
    f = GlacierFile(bytes(portable_container()))
    bulk = f.pages()
    assert [(e.page_id, e.data_offset, e.crc32) for e in bulk] == \
        [(f.page(i).page_id, f.page(i).data_offset, f.page(i).crc32) for i in range(f.num_pages)]
    count = ctypes.c_uint64()
    _lib.call("glacier_cuda_glacier_pages", f._ptr, f.size, None, 0, ctypes.byref(count))
    assert count.value == 2


@pytest.mark.parametrize("page_elems", [65536, 4096])
def test_host_model_reassembles_the_written_model(page_elems):
    """The host view of a file holds exactly the tensors it was written from, so tensor-parallel
    shards cut from the file equal the shards cut from the model."""
    from glacier_b200.glacier_file import host_model
    from glacier_b200.model import ModelConfig, SyntheticModel, TensorParallelShard
    cfg = ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)
    m = SyntheticModel(cfg, seed=9)
    ov = dict(num_heads=8, num_kv_heads=2, head_dim=64, eps=cfg.eps, theta=cfg.theta)
    hm = host_model(GlacierFile(bytes(gw.model_image(m, page_elems=page_elems))), ov)
    assert hm.cfg == m.cfg
    assert hm.embedding.dtype == np.float16 and np.array_equal(hm.embedding, m.embedding)
    assert np.array_equal(hm.final_norm, m.final_norm)
    for a, b in zip(hm.lm_head, m.lm_head):
        assert np.array_equal(a, b)
    for La, Lb in zip(hm.layers, m.layers):
        for k, v in Lb.items():
            if isinstance(v, tuple):
                assert all(np.array_equal(x, y) for x, y in zip(La[k], v)), k
            else:
                assert np.array_equal(La[k], v), k
    sa, sb = TensorParallelShard(hm, 1, 2), TensorParallelShard(m, 1, 2)
    assert sa.cfg == sb.cfg
    for La, Lb in zip(sa.layers, sb.layers):
        for k, v in Lb.items():
            if isinstance(v, tuple):
                assert all(np.array_equal(x, y) for x, y in zip(La[k], v)), k


def test_host_model_tied_int4_embedding():
    from glacier_b200.glacier_file import host_model
    from glacier_b200.model import ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=1, dim=64, hidden=128, num_heads=4, num_kv_heads=2, head_dim=16, vocab=32)
    m = SyntheticModel(cfg, seed=2)
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, 32 * 64 // 2, dtype=np.uint8)
    scales = rng.random(32 * 64 // 32, dtype=np.float32)
    img = gw.model_image(m, embedding=("int4", packed, scales), tie=True)
    hm = host_model(GlacierFile(bytes(img)), dict(num_heads=4, num_kv_heads=2, head_dim=16,
                                                   tie_word_embeddings=True))
    q = np.stack([packed & 15, packed >> 4], -1).reshape(-1).astype(np.float32) - 7
    assert hm.embedding.dtype == np.float32
    assert np.array_equal(hm.embedding.ravel(), q * np.repeat(scales, 32))
    assert np.array_equal(hm.lm_head[0], packed) and np.array_equal(hm.lm_head[1], scales)
