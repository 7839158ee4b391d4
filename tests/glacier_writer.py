"""Test-side writer of `.glacier` images (src/model/format.zig Header.writeTo
:84-101, PageEntry.writeTo :153-167; qio.zig encodePage :73-113).

It writes with Python's struct and zlib.crc32, independently of the library
under test, so the reader is checked against a second implementation of the
format.  Models are written the way the reference converter lays them out:
INT4 tensors in pages of at most 65536 elements, every page but a tensor's
last covering whole groups, each page carrying its own groups' scales.
"""
from __future__ import annotations

import json
import struct
import zlib

import numpy as np

HEADER_SIZE = 256
ENTRY_SIZE = 64
QIO_MAGIC = 0x514F4954

KIND = dict(embedding=0, attn_q=1, attn_k=2, attn_v=3, attn_o=4, mlp_up=5, mlp_down=6, mlp_gate=7, input_norm=8,
            lm_head=9, final_norm=10, post_attn_norm=11, attn_q_bias=12, attn_k_bias=13, attn_v_bias=14,
            attn_o_bias=15, other=255)
PREC = dict(fp16=0, bf16=1, int8=2, int4=3, int2=4, tri1p58=5, fp32=6)


def header_bytes(meta_len: int, num_pages: int, version: int = 1, page_size_log2: int = 18) -> bytearray:
    index_off = HEADER_SIZE + meta_len
    h = bytearray(HEADER_SIZE)
    struct.pack_into("<4sHHQQQQQII", h, 0, b"GLAC", version, HEADER_SIZE, HEADER_SIZE, meta_len, num_pages,
                     index_off, index_off + num_pages * ENTRY_SIZE, page_size_log2, 0)
    return h


def entry_bytes(page_id, layer, kind, row_start, row_end, precision, group, crc, offset, length) -> bytes:
    return struct.pack("<QIIQQBBHQQIII", page_id, layer, kind, row_start, row_end, precision, group, 0, offset,
                       length, crc, 0, 0)


def qio_payload(num_elements: int, group: int, precision: int, scales, packed) -> bytes:
    """16-byte sub-header (magic, elements, group, precision byte 0 int8 / 1 int4), scales, codes."""
    sub = struct.pack("<IIIB3x", QIO_MAGIC, num_elements, group, precision)
    return sub + np.ascontiguousarray(scales, np.float32).tobytes() + np.ascontiguousarray(packed, np.uint8).tobytes()


class Page:
    def __init__(self, layer, kind, row_start, row_end, precision, group, payload):
        self.layer, self.kind, self.row_start, self.row_end = layer, kind, row_start, row_end
        self.precision, self.group, self.payload = precision, group, payload


def build(pages: list[Page], metadata: str | bytes = '{"format":"test"}') -> bytearray:
    meta = metadata.encode() if isinstance(metadata, str) else metadata
    out = header_bytes(len(meta), len(pages))
    out += meta
    off = HEADER_SIZE + len(meta) + ENTRY_SIZE * len(pages)
    for i, p in enumerate(pages):
        out += entry_bytes(i, p.layer, p.kind, p.row_start, p.row_end, p.precision, p.group,
                           zlib.crc32(p.payload), off, len(p.payload))
        off += len(p.payload)
    for p in pages:
        out += p.payload
    return out


def int4_pages(layer: int, kind: str, packed, scales, group: int, page_elems: int = 65536) -> list[Page]:
    """One INT4 tensor (flat codes, flat group scales) cut into pages of whole groups."""
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    n = packed.size * 2
    assert page_elems % group == 0 and page_elems % 2 == 0
    pages = []
    for lo in range(0, n, page_elems):
        hi = min(n, lo + page_elems)
        g0, g1 = lo // group, -(-hi // group)
        pages.append(Page(layer, KIND[kind], lo, hi, PREC["int4"], group,
                          qio_payload(hi - lo, group, 1, scales[g0:g1], packed[lo // 2:hi // 2])))
    return pages


def raw_pages(layer: int, kind: str, values, precision: str = "fp32") -> list[Page]:
    """A raw tensor in pages of at most 256 KiB."""
    dt = {"fp32": np.float32, "fp16": np.float16}.get(precision)
    if precision == "bf16":
        a = np.ascontiguousarray(values, np.float32).reshape(-1)
        data = (a.view(np.uint32) >> 16).astype(np.uint16)
        esize = 2
    else:
        data = np.ascontiguousarray(values, dt).reshape(-1)
        esize = data.itemsize
    per = (1 << 18) // esize
    return [Page(layer, KIND[kind], lo, min(data.size, lo + per), PREC[precision], 0,
                 data[lo:lo + per].tobytes()) for lo in range(0, data.size, per)]


def model_image(m, embedding: str = "fp16", tie: bool = False, lm_head_pages: bool = True,
                page_elems: int = 65536, extra: list[Page] | None = None, drop: tuple = ()) -> bytearray:
    """A synthetic model (glacier_b200.model.SyntheticModel layout) as a `.glacier` image.

    ``embedding`` is "fp16" (the model's table), "bf16"/"fp32" (the same values
    widened) or ("int4", packed, scales) for an INT4 table.  ``drop`` names
    (layer, kind) groups to leave out.
    """
    c = m.cfg
    g = c["group"]
    pages: list[Page] = []

    def add(ps):
        pages.extend(p for p in ps if (p.layer, p.kind) not in {(l, KIND[k]) for l, k in drop})

    if isinstance(embedding, tuple):
        add(int4_pages(0, "embedding", embedding[1], embedding[2], g, page_elems))
    else:
        add(raw_pages(0, "embedding", np.asarray(m.embedding, np.float32), embedding))
    for i, L in enumerate(m.layers):
        for key, kind in (("wq", "attn_q"), ("wk", "attn_k"), ("wv", "attn_v"), ("wo", "attn_o"),
                          ("wg", "mlp_gate"), ("wu", "mlp_up"), ("wd", "mlp_down")):
            add(int4_pages(i, kind, *L[key], g, page_elems))
        add(raw_pages(i, "input_norm", L["input_norm"]))
        add(raw_pages(i, "post_attn_norm", L["post_attn_norm"]))
        for key, kind in (("bq", "attn_q_bias"), ("bk", "attn_k_bias"), ("bv", "attn_v_bias")):
            if L.get(key) is not None:
                add(raw_pages(i, kind, L[key]))
    add(raw_pages(0, "final_norm", m.final_norm))
    if lm_head_pages and not tie:
        add(int4_pages(0, "lm_head", *m.lm_head, g, page_elems))
    pages.extend(extra or [])
    meta = json.dumps({"schema": "glacier.model-conversion/v1", "architecture": "qwen2",
                       "tie_word_embeddings": tie})
    return build(pages, meta)
