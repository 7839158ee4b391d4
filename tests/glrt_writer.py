"""Test-side writer of prepared runtime images (`.glrt`), following
docs/RUNTIME_IMAGE.md and src/model/runtime_image.zig (Header.encode :227-256,
Record.encode :354-381, the canonical stream order and 64-byte alignment).

Python's struct, zlib.crc32 and hashlib.sha256 do the encoding, so the
library's reader is checked against an independent implementation.  The
layout helpers restate int4_weights.zig: rows4_k16 nibble order
(packedNibbleIndex :153-170), the rows4 fp16 scale grid (withRows4F16Scales
:362-386) and PairNibble pairing (pairRows4K16 :251-346).
"""
from __future__ import annotations

import hashlib
import struct
import zlib

import numpy as np

import glacier_writer as gw

HEADER, REC_V1, REC_V2, ALIGN = 512, 128, 160, 64
GLOBAL = 0xFFFFFFFF
STREAMS = ("packed", "f32", "f16", "rows4", "raw")
ABI = {  # (version, policy) -> execution-ABI fingerprint listed in docs/RUNTIME_IMAGE.md
    (1, "portable"): "0c1f185ceff5e9d366a920c8b0046f1543290f85965fbd7cb13f21fe2eec42b6",
    (1, "aarch64"): "dc5fe778a28150235c6f11c53bbf876e130dde0804c3b7a492f4de7e059bc7ad",
    (2, "portable"): "8f291472be36fab2d8e32bfbb87671ebbb18a982036a2d17dc06cbe2907ec890",
    (2, "aarch64"): "d0d7df06350af6b2d48e282f65ff873a3cf95bd6397b1d2d26cc6e679304e06f",
}


def rows4_index(row, col, in_f):
    return (row // 4) * (4 * in_f) + (col // 16) * 64 + ((col % 16) // 4) * 16 + (row % 4) * 4 + col % 4


def nibbles(packed, n):
    return np.stack([packed & 15, packed >> 4], -1).reshape(-1)[:n].astype(np.uint8)


def pack(nib):
    nib = np.asarray(nib, np.uint8)
    if nib.size % 2:
        nib = np.append(nib, 0)
    return (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8)


def rows4_perm(out_f, in_f):
    """perm[logical row-major index] = physical rows4_k16 nibble index."""
    r, c = np.meshgrid(np.arange(out_f), np.arange(in_f), indexing="ij")
    return rows4_index(r, c, in_f).reshape(-1)


def to_rows4(packed, out_f, in_f):
    nib = nibbles(packed, out_f * in_f)
    phys = np.zeros_like(nib)
    phys[rows4_perm(out_f, in_f)] = nib
    return pack(phys)


def rows4_grid(scales_f32, out_f):
    """Row-major group scales -> [tile][group][lane] fp16 grid."""
    per = scales_f32.size // out_f
    s = np.asarray(scales_f32, np.float32).reshape(out_f // 4, 4, per)
    return s.transpose(0, 2, 1).reshape(-1).astype(np.float16)


def pair(gate_packed, up_packed, gate_scales, up_scales, out_f, in_f):
    """PairNibble bytes (gate low, up high, rows4 order) and the [tile][group][branch][lane] scale grid."""
    perm = rows4_perm(out_f, in_f)
    g = np.zeros(out_f * in_f, np.uint8)
    u = np.zeros(out_f * in_f, np.uint8)
    g[perm] = nibbles(gate_packed, out_f * in_f)
    u[perm] = nibbles(up_packed, out_f * in_f)
    gg = rows4_grid(gate_scales, out_f).reshape(-1, 4)
    ug = rows4_grid(up_scales, out_f).reshape(-1, 4)
    return (g | (u << 4)).astype(np.uint8), np.concatenate([gg, ug], 1).reshape(-1)


class Rec:
    def __init__(self, layer, kind, encoding, layout, group, out_f, in_f, streams, role=0, pair_layout=0xFFFF,
                 flags=0):
        self.layer, self.kind, self.encoding, self.layout = layer, kind, encoding, layout
        self.group, self.out_f, self.in_f, self.role, self.pair_layout = group, out_f, in_f, role, pair_layout
        self.flags = flags
        self.streams = {k: bytes(np.ascontiguousarray(v).tobytes()) for k, v in streams.items()}


def raw_rec(layer, kind, values):
    v = np.asarray(values, np.float32).reshape(-1)
    return Rec(layer, gw.KIND[kind], 0, 0xFFFF, 0, 1, v.size, {"raw": v})


def int4_rec(layer, kind, packed, scales, out_f, in_f, group, layout="row_major", scale_streams=("f32",)):
    streams = {"packed": packed if layout == "row_major" else to_rows4(packed, out_f, in_f)}
    scales = np.asarray(scales, np.float32)
    if "f32" in scale_streams:
        streams["f32"] = scales
    if "f16" in scale_streams:
        streams["f16"] = scales.astype(np.float16)
    if "rows4" in scale_streams:
        streams["rows4"] = rows4_grid(scales, out_f)
    return Rec(layer, gw.KIND[kind], 1, {"row_major": 0, "rows4_k16": 1}[layout], group, out_f, in_f, streams)


def pair_rec(layer, gate, up, out_f, in_f, group):
    pb, ps = pair(gate[0], up[0], gate[1], up[1], out_f, in_f)
    return Rec(layer, gw.KIND["mlp_gate"], 2, 0xFFFF, group, out_f, in_f, {"packed": pb, "rows4": ps}, role=1,
               pair_layout=0)


def align(x):
    return -(-x // ALIGN) * ALIGN


def encode_record(r: Rec, version, offsets, crc, digest=b"\0" * 32):
    out = bytearray(REC_V2 if version == 2 else REC_V1)
    n = r.out_f * r.in_f
    struct.pack_into("<IIHHIIIIIQ", out, 0, r.layer, r.kind, r.encoding, r.layout, r.group, r.out_f, r.in_f,
                     r.flags, crc, n)
    for i, (off, ln) in enumerate(offsets):
        struct.pack_into("<QQ", out, 40 + 16 * i, off, ln)
    if version == 2:
        struct.pack_into("<HH", out, 120, r.role, r.pair_layout)
        out[128:160] = digest
    return out


def build(recs, cfg: dict, version=2, policy="portable", source_fp=b"\x11" * 32, mutate_record=None) -> bytearray:
    """cfg: dim, hidden, layers, vocab, heads, head_dim, kv_heads, eps, theta, tie."""
    rsize = REC_V2 if version == 2 else REC_V1
    data_off = align(HEADER + rsize * len(recs))
    body = bytearray()
    index = bytearray()
    pos = data_off
    for r in recs:
        offsets = []
        payload = b""
        for name in STREAMS:
            blob = r.streams.get(name, b"")
            if not blob:
                offsets.append((0, 0))
                continue
            pad = align(pos) - pos
            body += b"\0" * pad
            pos += pad
            offsets.append((pos, len(blob)))
            body += blob
            pos += len(blob)
            payload += blob
        crc = zlib.crc32(payload)
        desc = encode_record(r, version, offsets, crc)
        if version == 2:
            desc[128:160] = hashlib.sha256(bytes(desc[:128]) + payload).digest()
        if mutate_record:
            mutate_record(r, desc)
        index += desc
    file_size = align(pos)
    body += b"\0" * (file_size - pos)
    h = bytearray(HEADER)
    struct.pack_into("<4sHHHHIQQQQ", h, 0, b"GLRT", version, HEADER, rsize, ALIGN, 0, len(recs), HEADER, data_off,
                     file_size)
    h[48:80] = source_fp
    h[80:112] = bytes.fromhex(ABI[(version, policy)])
    struct.pack_into("<7IB", h, 112, cfg["dim"], cfg["hidden"], cfg["layers"], cfg["vocab"], cfg["heads"],
                     cfg["head_dim"], cfg["kv_heads"], int(cfg["tie"]))
    struct.pack_into("<ff", h, 144, cfg["eps"], cfg["theta"])
    struct.pack_into("<I", h, 152, zlib.crc32(bytes(index)))
    struct.pack_into("<I", h, 156, zlib.crc32(bytes(h)))
    out = h + index + b"\0" * (data_off - HEADER - len(index)) + body[0:]
    # body began at data_off
    assert len(out) == file_size, (len(out), file_size)
    return out


def refresh_crcs(img: bytearray, version=2):
    """Recompute the index and header CRCs after a test edited the index."""
    count = struct.unpack_from("<Q", img, 16)[0]
    rsize = REC_V2 if version == 2 else REC_V1
    struct.pack_into("<I", img, 152, zlib.crc32(bytes(img[HEADER:HEADER + count * rsize])))
    struct.pack_into("<I", img, 156, 0)
    struct.pack_into("<I", img, 156, zlib.crc32(bytes(img[:HEADER])))
    return img


def model_cfg(m, tie=False):
    c = m.cfg
    return dict(dim=c["dim"], hidden=c["hidden"], layers=c["num_layers"], vocab=c["vocab"], heads=c["num_heads"],
                head_dim=c["head_dim"], kv_heads=c["num_kv_heads"], eps=c["eps"], theta=c["theta"], tie=tie)


def model_records(m, embedding, layout="row_major", scale_streams=("f32",), mlp="separate", tie=False):
    """Records of a SyntheticModel; embedding is (packed, scales_f32) INT4 data."""
    c = m.cfg
    D, F, KV, g = c["dim"], c["hidden"], c["num_kv_heads"] * c["head_dim"], c["group"]
    recs = []
    for i, L in enumerate(m.layers):
        recs.append(raw_rec(i, "input_norm", L["input_norm"]))
        for key, kind in (("bq", "attn_q_bias"), ("bk", "attn_k_bias"), ("bv", "attn_v_bias")):
            recs.append(raw_rec(i, kind, L[key]))
        recs.append(raw_rec(i, "post_attn_norm", L["post_attn_norm"]))
        for key, kind, o, k in (("wq", "attn_q", D, D), ("wk", "attn_k", KV, D), ("wv", "attn_v", KV, D),
                                ("wo", "attn_o", D, D), ("wd", "mlp_down", D, F)):
            recs.append(int4_rec(i, kind, *L[key], o, k, g, layout, scale_streams))
        if mlp == "pair":
            recs.append(pair_rec(i, L["wg"], L["wu"], F, D, g))
        else:
            recs.append(int4_rec(i, "mlp_gate", *L["wg"], F, D, g, layout, scale_streams))
            recs.append(int4_rec(i, "mlp_up", *L["wu"], F, D, g, layout, scale_streams))
    recs.append(raw_rec(GLOBAL, "final_norm", m.final_norm))
    emb_streams = tuple(sorted(set(scale_streams) | {"f32"}))
    recs.append(int4_rec(GLOBAL, "embedding", *embedding, c["vocab"], D, g, layout, emb_streams))
    if not tie:
        recs.append(int4_rec(GLOBAL, "lm_head", *m.lm_head, c["vocab"], D, g, layout, scale_streams))
    return recs
