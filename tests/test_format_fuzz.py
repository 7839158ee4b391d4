"""Hostile-file robustness of the two readers (host code, no GPU).

Seeded random mutations of valid images (byte flips in the header, metadata
and index, random truncations and extensions) must each end in a clean
GLACIER_CUDA_EFORMAT or a successful admission: never a crash, hang or read
outside the buffer.  The reference's readers make the same promise with
checked arithmetic for every offset (format.zig:216-345,
runtime_image.zig:432-590).
"""
import numpy as np
import pytest

import glacier_writer as gw
import glrt_writer as gr
from glacier_b200 import _lib
from glacier_b200.glacier_file import GlacierFile
from glacier_b200.runtime_image import RuntimeImage


def small_model():
    from glacier_b200.model import ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=1, dim=64, hidden=128, num_heads=4, num_kv_heads=2, head_dim=16, vocab=32, group=16)
    return SyntheticModel(cfg, seed=4)


def mutations(img: bytes, head: int, rng, n: int):
    for _ in range(n):
        b = bytearray(img)
        kind = rng.integers(0, 4)
        if kind < 2:  # flip 1-4 bytes in the structural prefix
            for _ in range(int(rng.integers(1, 5))):
                b[int(rng.integers(0, min(head, len(b))))] ^= int(rng.integers(1, 256))
        elif kind == 2:
            del b[int(rng.integers(0, len(b))):]
        else:
            b += bytes(int(rng.integers(1, 200)))
        yield bytes(b)


def exercise_glacier(data: bytes):
    try:
        f = GlacierFile(data)
    except _lib.GlacierCudaError as e:
        assert e.code == _lib.EFORMAT
        return
    for call in (f.validate_pages, f.pages, f.geometry):
        try:
            call()
        except _lib.GlacierCudaError as e:
            assert e.code == _lib.EFORMAT
    for i in range(min(f.num_pages, 4)):
        try:
            f.decode_page(i)
        except _lib.GlacierCudaError as e:
            assert e.code == _lib.EFORMAT


def exercise_glrt(data: bytes):
    try:
        r = RuntimeImage(data)
    except _lib.GlacierCudaError as e:
        assert e.code == _lib.EFORMAT
        return
    r.records()
    try:
        r.model_info()
    except _lib.GlacierCudaError as e:
        assert e.code in (_lib.EFORMAT, _lib.EUNSUPPORTED)


def test_glacier_reader_survives_mutations():
    img = bytes(gw.model_image(small_model()))
    f = GlacierFile(img)
    head = int(f.info.page_data_offset) + 64
    rng = np.random.default_rng(11)
    for data in mutations(img, head, rng, 400):
        exercise_glacier(data)


def test_glrt_reader_survives_mutations():
    m = small_model()
    rng = np.random.default_rng(12)
    emb = (rng.integers(0, 256, 32 * 64 // 2, dtype=np.uint8), (rng.integers(1, 16, 32 * 64 // 16) / 256).astype(np.float32))
    img = bytes(gr.build(gr.model_records(m, emb, mlp="pair"), gr.model_cfg(m)))
    head = int(RuntimeImage(img).info.data_offset) + 64
    for data in mutations(img, head, rng, 400):
        exercise_glrt(data)


@pytest.mark.parametrize("n", [0, 1, 255, 256, 511, 512])
def test_tiny_inputs(n):
    for data in (bytes(n), b"GLAC" + bytes(max(0, n - 4)), b"GLRT" + bytes(max(0, n - 4))):
        exercise_glacier(data)
        exercise_glrt(data)
