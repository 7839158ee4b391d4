"""A model loaded from a `.glacier` image decodes exactly like the same weights
uploaded tensor by tensor (loader.zig loadWithOptions :1214-1540 feeding
generate.zig's decode), and the loader's rejections surface before anything
runs.

The direct upload is itself checked against the CPU oracle by
test_gpu_decode.py, so bit-identical logits here carry that parity over to the
file path.  Images come from tests/glacier_writer.py.
"""
import copy
import json
import struct
import zlib

import numpy as np
import pytest

import glacier_writer as gw
from glacier_b200 import _lib
from glacier_b200.glacier_file import GlacierFile, load_model, reason_name

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_PAGES = 2


def small_cfg(group=32):
    from glacier_b200.model import ModelConfig
    return ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000,
                       group=group)


def overrides(cfg, tie=False):
    return dict(num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, eps=cfg.eps,
                theta=cfg.theta, tie_word_embeddings=tie)


def decode_logits(dm, lanes=2, steps=6, seed=11):
    """Logits of `steps` decode steps over fixed random tokens."""
    from glacier_b200.model import DecodeSession
    sess = DecodeSession(dm, lanes, MAX_PAGES)
    rng = np.random.default_rng(seed)
    toks = rng.integers(0, dm.cfg["vocab"], size=(steps, lanes)).astype(np.int32)
    lg = torch.empty((lanes, dm.cfg["vocab"]), dtype=torch.float32, device="cuda")
    out = []
    for pos in range(steps):
        sess.step(tokens=toks[pos], positions=[pos] * lanes, logits=lg)
        out.append(lg.cpu().numpy().copy())
        assert sess.status.cpu().numpy().tolist() == [0] * lanes
    sess.close()
    return np.stack(out)


def same_bits(a, b):
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("page_elems", [65536, 4096])
def test_glacier_load_matches_direct_upload(page_elems):
    from glacier_b200.model import DeviceModel, SyntheticModel
    cfg = small_cfg()
    m = SyntheticModel(cfg, seed=21)
    img = bytes(gw.model_image(m, page_elems=page_elems))
    gf = GlacierFile(img)
    assert gf.geometry().vocab == cfg.vocab
    fm = load_model(gf, MAX_PAGES * 16, overrides(cfg))
    dm = DeviceModel(m, MAX_PAGES * 16)
    try:
        assert same_bits(decode_logits(fm), decode_logits(dm))
    finally:
        fm.close()
        dm.close()


def short_significand_int4(rng, vocab, dim, group):
    """An INT4 table whose dequantized values are fp16-exact: scales m * 2^-e with m < 16."""
    packed = rng.integers(0, 256, size=vocab * dim // 2, dtype=np.uint8)
    m = rng.integers(1, 16, size=vocab * dim // group).astype(np.float32)
    scales = m * np.float32(2.0 ** -8)
    return packed, scales


def dequant(packed, scales, group):
    q = np.stack([packed & 15, packed >> 4], -1).reshape(-1).astype(np.float32) - 7
    return q * np.repeat(scales, group)


def test_tied_int4_embedding():
    """tie_word_embeddings: the LM head is the INT4 embedding (loader.zig:1521-1523), and the
    embedding lookup dequantizes rows in f32 (int4_matmul.zig dequantizeRow)."""
    from glacier_b200.model import DeviceModel, SyntheticModel
    cfg = small_cfg()
    m = SyntheticModel(cfg, seed=22)
    packed, scales = short_significand_int4(np.random.default_rng(1), cfg.vocab, cfg.dim, cfg.group)
    table = dequant(packed, scales, cfg.group).reshape(cfg.vocab, cfg.dim)
    assert np.array_equal(table.astype(np.float16).astype(np.float32), table)
    img = bytes(gw.model_image(m, embedding=("int4", packed, scales), tie=True))
    m2 = copy.copy(m)
    m2.embedding = table.astype(np.float16)
    m2.lm_head = (packed, scales)
    fm = load_model(GlacierFile(img), MAX_PAGES * 16, overrides(cfg, tie=True))
    dm = DeviceModel(m2, MAX_PAGES * 16)
    try:
        assert same_bits(decode_logits(fm), decode_logits(dm))
    finally:
        fm.close()
        dm.close()


def test_bf16_embedding_pages():
    """A bf16 table widens to f32 rows; values that bf16 and fp16 both hold decode identically."""
    from glacier_b200.model import DeviceModel, SyntheticModel
    cfg = small_cfg()
    m = SyntheticModel(cfg, seed=23)
    e = np.asarray(m.embedding, np.float32)
    e = (e.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)  # bf16-exact
    e = e.astype(np.float16).astype(np.float32)
    m.embedding = e.astype(np.float16)
    img = bytes(gw.model_image(m, embedding="bf16"))
    fm = load_model(GlacierFile(img), MAX_PAGES * 16, overrides(cfg))
    dm = DeviceModel(m, MAX_PAGES * 16)
    try:
        assert same_bits(decode_logits(fm), decode_logits(dm))
    finally:
        fm.close()
        dm.close()


def test_path_and_sidecar(tmp_path):
    """load_model(path) reads `<path>.json` (config.loadSidecar) for heads, eps and theta."""
    from glacier_b200.model import DeviceModel, SyntheticModel
    cfg = small_cfg()
    m = SyntheticModel(cfg, seed=24)
    path = tmp_path / "m.glacier"
    path.write_bytes(bytes(gw.model_image(m)))
    (tmp_path / "m.glacier.json").write_text(json.dumps({
        "num_attention_heads": cfg.num_heads, "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
        "rms_norm_eps": cfg.eps, "rope_theta": cfg.theta}))
    fm = load_model(str(path), MAX_PAGES * 16)
    dm = DeviceModel(m, MAX_PAGES * 16)
    try:
        assert fm.cfg["num_kv_heads"] == cfg.num_kv_heads and fm.cfg["theta"] == cfg.theta
        assert same_bits(decode_logits(fm), decode_logits(dm))
    finally:
        fm.close()
        dm.close()


def load_error(img, cfg, tie=False):
    with pytest.raises(_lib.GlacierCudaError) as e:
        load_model(GlacierFile(bytes(img)), MAX_PAGES * 16, overrides(cfg, tie))
    return e.value


def test_loader_rejections():
    from glacier_b200.model import SyntheticModel
    cfg = small_cfg()
    m = SyntheticModel(cfg, seed=25)
    err = load_error(gw.model_image(m, drop=((1, "mlp_down"),)), cfg)
    assert reason_name(err) == "MissingTensor" and "mlp_down" in str(err)
    err = load_error(gw.model_image(m, drop=((0, "post_attn_norm"),)), cfg)
    assert reason_name(err) == "MissingTensor"
    err = load_error(gw.model_image(m, lm_head_pages=False), cfg)
    assert reason_name(err) == "MissingTensor" and "lm_head" in str(err)
    # A tied head needs INT4 embedding data; the model has no dense LM-head path.
    assert load_error(gw.model_image(m, tie=True), cfg, tie=True).code == _lib.EUNSUPPORTED
    # Attention output bias: not part of the Qwen2 decode path the model implements.
    bo = gw.raw_pages(0, "attn_o_bias", np.zeros(cfg.dim, np.float32))
    assert load_error(gw.model_image(m, extra=bo), cfg).code == _lib.EUNSUPPORTED
    # One payload byte changed: CRC mismatch before any upload.
    img = gw.model_image(m)
    gf = GlacierFile(bytes(img))
    img[gf.page(gf.num_pages - 1).data_offset] ^= 1
    assert reason_name(load_error(img, cfg)) == "CrcMismatch"
    # A sub-header that disagrees with its entry under a valid CRC: readPage passes it and the
    # loader rejects the page (loader.zig:1697-1700).
    img = gw.model_image(m)
    last = gf.page(gf.num_pages - 1)
    struct.pack_into("<I", img, last.data_offset + 8, 16)  # group 16 in the sub-header, 32 in the entry
    payload = bytes(img[last.data_offset:last.data_offset + last.data_len])
    struct.pack_into("<I", img, gf.info.page_index_offset + 64 * (gf.num_pages - 1) + 52, zlib.crc32(payload))
    assert reason_name(load_error(img, cfg)) == "BadPayload"
    # A packed tensor whose non-final page splits a group (concatInt4Pages BadPayload).
    pk, sc = m.layers[0]["wq"]
    bad = gw.int4_pages(0, "attn_q", pk, sc, cfg.group)
    bad[0] = gw.Page(0, gw.KIND["attn_q"], 0, 48, gw.PREC["int4"], 32, gw.qio_payload(48, 32, 1, sc[:2], pk[:24]))
    err = load_error(gw.model_image(m, drop=((0, "attn_q"),), extra=bad), cfg)
    assert reason_name(err) == "BadPayload"


def test_group_16_image():
    """A group-16 file (the reference's aarch64 production layout) loads into a group-16 model."""
    from glacier_b200.model import DeviceModel, SyntheticModel
    cfg = small_cfg(group=16)
    m = SyntheticModel(cfg, seed=26)
    fm = load_model(GlacierFile(bytes(gw.model_image(m))), MAX_PAGES * 16, overrides(cfg))
    dm = DeviceModel(m, MAX_PAGES * 16)
    try:
        assert same_bits(decode_logits(fm), decode_logits(dm))
    finally:
        fm.close()
        dm.close()


def test_host_model_upload_matches_file_load():
    """A model uploaded tensor by tensor from the host view of a file (the path tensor-parallel
    shards take) decodes exactly like the library's own file loader, f32 embedding rows included."""
    from glacier_b200.glacier_file import host_model
    from glacier_b200.model import DeviceModel, SyntheticModel
    cfg = small_cfg()
    m = SyntheticModel(cfg, seed=27)
    rng = np.random.default_rng(5)
    packed = rng.integers(0, 256, cfg.vocab * cfg.dim // 2, dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(cfg.vocab * cfg.dim // cfg.group)) * 0.05).astype(np.float32)
    gf = GlacierFile(bytes(gw.model_image(m, embedding=("int4", packed, scales), tie=True)))
    ov = overrides(cfg, tie=True)
    fm = load_model(gf, MAX_PAGES * 16, ov)
    hm = DeviceModel(host_model(gf, ov), MAX_PAGES * 16)
    try:
        assert same_bits(decode_logits(fm), decode_logits(hm))
    finally:
        fm.close()
        hm.close()
