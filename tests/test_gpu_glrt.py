"""A model loaded from a prepared runtime image (`.glrt`) decodes exactly like
the same weights uploaded tensor by tensor, for every prepared layout: row-major
INT4 with f32 or fp16 scales, rows4_k16 codes with only the rows4 fp16 scale
grid (the reference's AArch64 preparation), PairNibble gate/up records, v1
images and a tied head (loader.zig loadPreparedOwnedFileWithOptionsV1
:216-385).  The direct upload is checked against the CPU oracle by
test_gpu_decode.py, so bit-identical logits carry that parity over.
"""
import copy

import numpy as np
import pytest

import glrt_writer as gr
from glacier_b200 import _lib
from glacier_b200.glacier_file import reason_name
from glacier_b200.runtime_image import RuntimeImage, load_model

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_PAGES = 2


def model(group=16, seed=31):
    from glacier_b200.model import ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=4, num_kv_heads=2, head_dim=64, vocab=1000,
                      group=group)
    m = SyntheticModel(cfg, seed=seed)
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, cfg.vocab * cfg.dim // 2, dtype=np.uint8)
    scales = (rng.integers(1, 16, cfg.vocab * cfg.dim // group) * 2.0 ** -8).astype(np.float32)
    return m, (packed, scales)


def direct_twin(m, emb, tie):
    """The SyntheticModel the prepared image describes: INT4 embedding rows (fp16-exact by
    construction) as its fp16 table, and the embedding's INT4 data as the head when tied."""
    m2 = copy.copy(m)
    q = gr.nibbles(emb[0], emb[0].size * 2).astype(np.float32) - 7
    table = (q * np.repeat(emb[1], m.cfg["group"])).reshape(m.cfg["vocab"], m.cfg["dim"])
    assert np.array_equal(table.astype(np.float16).astype(np.float32), table)
    m2.embedding = table.astype(np.float16)
    if tie:
        m2.lm_head = emb
    return m2


def decode_logits(dm, lanes=2, steps=5, seed=12):
    from glacier_b200.model import DecodeSession
    sess = DecodeSession(dm, lanes, MAX_PAGES)
    toks = np.random.default_rng(seed).integers(0, dm.cfg["vocab"], size=(steps, lanes)).astype(np.int32)
    lg = torch.empty((lanes, dm.cfg["vocab"]), dtype=torch.float32, device="cuda")
    out = []
    for pos in range(steps):
        sess.step(tokens=toks[pos], positions=[pos] * lanes, logits=lg)
        out.append(lg.cpu().numpy().copy())
        assert sess.status.cpu().numpy().tolist() == [0] * lanes
    sess.close()
    return np.stack(out)


@pytest.mark.parametrize("kw", [
    dict(),
    dict(scale_streams=("f16",)),
    dict(layout="rows4_k16", scale_streams=("rows4",)),
    dict(mlp="pair"),
    dict(layout="rows4_k16", scale_streams=("rows4",), mlp="pair", tie=True),
    dict(version=1),
    dict(group=8, mlp="pair", layout="rows4_k16", scale_streams=("rows4",)),
])
def test_prepared_image_matches_direct_upload(kw):
    from glacier_b200.model import DeviceModel
    kw = dict(kw)
    version, tie, group = kw.pop("version", 2), kw.pop("tie", False), kw.pop("group", 16)
    m, emb = model(group)
    img = gr.build(gr.model_records(m, emb, tie=tie, **kw), gr.model_cfg(m, tie=tie), version=version)
    fm = load_model(bytes(img), MAX_PAGES * 16)
    dm = DeviceModel(direct_twin(m, emb, tie), MAX_PAGES * 16)
    try:
        a, b = decode_logits(fm), decode_logits(dm)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    finally:
        fm.close()
        dm.close()


def test_load_rejections():
    from glacier_b200.model import DeviceModel  # noqa: F401
    m, emb = model()
    recs = gr.model_records(m, emb)
    # An attention output bias is outside the Qwen2 decode path the model implements.
    bo = recs + [gr.raw_rec(0, "attn_o_bias", np.zeros(256, np.float32))]
    with pytest.raises(_lib.GlacierCudaError) as e:
        load_model(bytes(gr.build(bo, gr.model_cfg(m))), MAX_PAGES * 16)
    assert e.value.code == _lib.EUNSUPPORTED
    # A payload byte flipped: rejected at admission, before any upload.
    img = gr.build(recs, gr.model_cfg(m))
    r = RuntimeImage(bytes(img))
    img[r.record(3).stream_offset[4]] ^= 1
    with pytest.raises(_lib.GlacierCudaError) as e:
        load_model(bytes(img), MAX_PAGES * 16)
    assert reason_name(e.value) == "CrcMismatch"


def test_host_model_upload_matches_image_load():
    """Uploading the host view of a prepared image (the tensor-parallel path) decodes exactly like
    the library's own image loader, for a rows4_k16 PairNibble image with a tied head."""
    from glacier_b200.model import DeviceModel
    from glacier_b200.runtime_image import host_model
    m, emb = model()
    img = bytes(gr.build(gr.model_records(m, emb, tie=True, layout="rows4_k16", scale_streams=("rows4",),
                                          mlp="pair"), gr.model_cfg(m, tie=True)))
    fm = load_model(img, MAX_PAGES * 16)
    hm = DeviceModel(host_model(img), MAX_PAGES * 16)
    try:
        a, b = decode_logits(fm), decode_logits(hm)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    finally:
        fm.close()
        hm.close()
