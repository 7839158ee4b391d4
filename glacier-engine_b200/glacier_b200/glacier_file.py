"""The portable `.glacier` model container through the C ABI.

``GlacierFile`` admits an image the way the reference's ``FileReader.open``
does (src/model/format.zig:383-478) and gives page-level access;
``load_model`` builds a device-resident model from it the way
``loader.load`` does (src/loader.zig:1205-1540), with the optional
``<path>.json`` sidecar of ``config.loadSidecar`` (src/config.zig:46-92)
overriding the geometry the page metadata implies.  All parsing and
validation runs in the library (csrc/model_format.cu); this module only
holds the bytes and converts results.
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np

from . import _lib

# enum glacier_cuda_format_reason, by value: the reference error each code stands for.
REASONS = ("Ok", "TruncatedHeader", "BadMagic", "BadVersion", "BadHeaderSize", "BadPageSize", "BadReservedField",
           "BadLayout", "MetadataTooLarge", "IndexTooLarge", "LayoutOverflow", "TruncatedMeta", "TruncatedIndex",
           "BadMetadata", "BadTensorKind", "BadPrecision", "BadPageId", "BadRowRange", "EmptyPage", "BadQuantGroup",
           "PageGeometryTooLarge", "UnsupportedPrecision", "BadPageGeometry", "NonContiguousPayload",
           "TruncatedPage", "TrailingBytes", "BadQuantPayload", "CrcMismatch", "SizeMismatch", "NoLayers",
           "MissingTensor", "BadPayload", "BadRecordSize", "BadAlignment", "BadConfig", "HeaderCrcMismatch",
           "IndexCrcMismatch", "LegacyVersionDisabled", "BadHeader", "BadBounds", "SourceFingerprintMismatch",
           "AbiFingerprintMismatch", "BadEncoding", "BadPackedLayout", "BadRole", "BadPairNibbleLayout", "BadFlags",
           "BadVersionedRecord", "MissingDigest", "BadTensorShape", "MissingScales", "OverlappingPayload",
           "DuplicateRecord", "DigestMismatch")

# TensorKind (format.zig:44-62) and StoredPrecision (core/precision.zig:9-16).
TENSOR_KINDS = {0: "embedding", 1: "attn_q", 2: "attn_k", 3: "attn_v", 4: "attn_o", 5: "mlp_up", 6: "mlp_down",
                7: "mlp_gate", 8: "input_norm", 9: "lm_head", 10: "final_norm", 11: "post_attn_norm",
                12: "attn_q_bias", 13: "attn_k_bias", 14: "attn_v_bias", 15: "attn_o_bias", 255: "other"}
PRECISIONS = {0: "fp16", 1: "bf16", 2: "int8", 3: "int4", 4: "int2", 5: "tri1p58", 6: "fp32"}


def _map_file(path: str) -> np.ndarray:
    """The file as a read-only byte array: a memory mapping (pages load on first
    touch, nothing is copied), or an empty array for an empty file."""
    if os.path.getsize(path) == 0:
        return np.zeros(0, np.uint8)
    return np.memmap(path, dtype=np.uint8, mode="r")


def reason_name(err: _lib.GlacierCudaError) -> str:
    """The reference error name behind a GLACIER_CUDA_EFORMAT failure."""
    return REASONS[err.reason] if 0 <= err.reason < len(REASONS) else f"reason {err.reason}"


def crc32(data) -> int:
    buf = np.frombuffer(memoryview(data), np.uint8)
    return int(_lib.lib().glacier_cuda_crc32(buf.ctypes.data if buf.size else None, buf.size))


class GlacierFile:
    """An admitted `.glacier` image held in host memory (read once, or a file mapping)."""

    def __init__(self, source):
        if isinstance(source, (str, os.PathLike)):
            self.path = os.fspath(source)
            self._buf = _map_file(self.path)
        else:
            self.path = None
            self._buf = np.frombuffer(memoryview(source), np.uint8)
        self.info = _lib.FileInfo()
        _lib.call("glacier_cuda_glacier_open", self._ptr, self.size, C.byref(self.info))

    @property
    def _ptr(self):
        return self._buf.ctypes.data if self._buf.size else None

    @property
    def size(self) -> int:
        return int(self._buf.size)

    @property
    def num_pages(self) -> int:
        return int(self.info.num_pages)

    def metadata(self) -> dict:
        lo = self.info.meta_offset
        return json.loads(bytes(self._buf[lo:lo + self.info.meta_len]))

    def page(self, index: int) -> _lib.PageEntry:
        e = _lib.PageEntry()
        _lib.call("glacier_cuda_glacier_page", self._ptr, self.size, index, C.byref(e))
        return e

    def pages(self) -> list[_lib.PageEntry]:
        """Every page entry, from one admission of the image."""
        n = self.num_pages
        arr = (_lib.PageEntry * max(n, 1))()
        count = C.c_uint64()
        _lib.call("glacier_cuda_glacier_pages", self._ptr, self.size, arr, n, C.byref(count))
        return list(arr[:count.value])

    def validate_pages(self) -> None:
        """Every quantized sub-header and CRC-32 (FileReader.validateAllPageCrcs)."""
        _lib.call("glacier_cuda_glacier_validate_pages", self._ptr, self.size)

    def decode_page(self, index: int) -> np.ndarray:
        """One page's elements as float32 (FileReader.readPageDequant(f32))."""
        e = self.page(index)
        out = np.empty(e.row_end - e.row_start, np.float32)
        _lib.call("glacier_cuda_glacier_page_decode_f32", self._ptr, self.size, index, out.ctypes.data, out.size)
        return out

    def geometry(self) -> _lib.FileGeometry:
        g = _lib.FileGeometry()
        _lib.call("glacier_cuda_glacier_geometry", self._ptr, self.size, C.byref(g))
        return g


def parse_sidecar(text: str | bytes) -> dict:
    """config.zig parseJson (:66-92): the overrides a `<model>.json` sidecar sets.

    Sizes must be non-negative JSON integers, eps/theta integers or floats and
    the tie flag a boolean; any other value type leaves that field unset.
    """
    obj = json.loads(text)
    if not isinstance(obj, dict):
        raise ValueError("sidecar is not a JSON object")

    def usize(*keys):  # first key holding a valid value, as `a orelse b` does
        for k in keys:
            v = obj.get(k)
            if type(v) is int and v >= 0:
                return v
        return None

    def f32(*keys):
        for k in keys:
            v = obj.get(k)
            if type(v) in (int, float):
                return float(np.float32(v))
        return None

    out = {
        "dim": usize("dim", "hidden_size"),
        "hidden": usize("hidden_dim", "intermediate_size"),
        "num_layers": usize("num_layers", "num_hidden_layers"),
        "vocab": usize("vocab_size"),
        "num_heads": usize("num_heads", "num_attention_heads"),
        "head_dim": usize("head_dim"),
        "eps": f32("rms_eps", "rms_norm_eps"),
        "theta": f32("rope_theta"),
        "num_kv_heads": usize("num_kv_heads", "num_key_value_heads"),
        "tie_word_embeddings": obj.get("tie_word_embeddings") if type(obj.get("tie_word_embeddings")) is bool
        else None,
    }
    return {k: v for k, v in out.items() if v is not None}


def resolve_config(geometry: _lib.FileGeometry, overrides: dict) -> dict:
    """loader.zig:1525-1541: sidecar values over the page-metadata geometry.

    Defaults where neither gives a value: eps 1e-6, theta 10000, head_dim 64
    (dim itself when dim is not a multiple of 64), heads dim / head_dim, and as
    many KV heads as query heads.
    """
    dim = overrides.get("dim", geometry.dim)
    heads_default, hd_default = (dim // 64, 64) if dim >= 64 and dim % 64 == 0 else (1, dim)
    num_heads = overrides.get("num_heads", heads_default)
    return dict(num_layers=overrides.get("num_layers", geometry.num_layers), dim=dim,
                hidden=overrides.get("hidden", geometry.hidden), num_heads=num_heads,
                num_kv_heads=overrides.get("num_kv_heads", num_heads), head_dim=overrides.get("head_dim", hd_default),
                vocab=overrides.get("vocab", geometry.vocab), group=geometry.group_size,
                eps=overrides.get("eps", 1e-6), theta=overrides.get("theta", 10000.0),
                tie_word_embeddings=bool(overrides.get("tie_word_embeddings", False)))


def load_model(source, max_positions: int, overrides: dict | None = None, scales_f16: bool = True):
    """A finalized DeviceModel built from a `.glacier` image on the current device.

    ``source`` is a path (its ``<path>.json`` sidecar is read when present, as
    loadSidecar does) or a GlacierFile / bytes; ``overrides`` wins over both.
    """
    from .model import DeviceModel
    gf = source if isinstance(source, GlacierFile) else GlacierFile(source)
    ov = {}
    if gf.path and os.path.exists(gf.path + ".json"):
        with open(gf.path + ".json", "rb") as f:
            ov.update(parse_sidecar(f.read()))
    ov.update(overrides or {})
    cfg = resolve_config(gf.geometry(), ov)
    return DeviceModel.from_glacier(gf, cfg, max_positions, scales_f16)


class HostModel:
    """A `.glacier` model's tensors as host arrays, in the layout glacier_b200.model
    uses (layers of (packed, scales) INT4 pairs and f32 vectors), so that
    TensorParallelShard can cut a real file into per-GPU shards the same way it
    cuts a synthetic model.  Tensors are assembled as the library's loader does
    (loader.zig:1214-1540): INT4 pages concatenated in page order with their
    per-page scales, raw pages decoded to f32; an fp16 embedding stays fp16 and
    any other embedding becomes f32 rows (INT4 rows as dequantizeRow forms
    them); a tied head reuses the INT4 embedding."""

    KINDS = {1: "wq", 2: "wk", 3: "wv", 4: "wo", 5: "wu", 6: "wd", 7: "wg", 8: "input_norm", 11: "post_attn_norm",
             12: "bq", 13: "bk", 14: "bv"}

    def __init__(self, gf: GlacierFile, cfg: dict):
        from .model import ModelConfig
        self.cfg = {k: cfg[k] for k in ("num_layers", "dim", "hidden", "num_heads", "num_kv_heads", "head_dim",
                                        "vocab", "group", "eps", "theta")}
        self.config = ModelConfig(**self.cfg)
        gf.validate_pages()
        groups: dict = {}
        for e in gf.pages():
            groups.setdefault((e.layer_idx, e.tensor_kind), []).append(e)
        buf = gf._buf

        def int4(pages):
            g = pages[0].quant_group
            packed, scales = [], []
            for k, e in enumerate(pages):
                n = e.row_end - e.row_start
                if e.precision != 3 or e.quant_group != g or (k + 1 < len(pages) and (n % g or n % 2)):
                    raise ValueError(f"page {e.page_id}: not an INT4 page of whole groups")
                ng = -(-n // g)
                base = e.data_offset + 16
                scales.append(np.frombuffer(buf[base:base + 4 * ng].tobytes(), np.float32))
                packed.append(np.asarray(buf[base + 4 * ng:base + 4 * ng + -(-n // 2)]))
            return np.concatenate(packed).astype(np.uint8), np.concatenate(scales)

        def raw(pages):
            return np.concatenate([gf.decode_page(int(e.page_id)) for e in pages])

        self.layers = [dict() for _ in range(self.cfg["num_layers"])]
        for (layer, kind), pages in groups.items():
            name = self.KINDS.get(kind)
            if name is None or layer >= len(self.layers):
                continue
            self.layers[layer][name] = int4(pages) if name.startswith("w") else raw(pages)
        for i, L in enumerate(self.layers):
            for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "input_norm", "post_attn_norm"):
                if name not in L:
                    raise ValueError(f"layer {i} has no {name}")
            for name in ("bq", "bk", "bv"):
                L.setdefault(name, None)
        for key, what in (((0, 10), "final norm"), ((0, 0), "embedding")):
            if key not in groups:
                raise ValueError(f"the model has no {what} tensor")
        if not cfg.get("tie_word_embeddings") and (0, 9) not in groups:
            raise ValueError("the model has no LM head tensor and does not tie it to the embedding")
        self.final_norm = raw(groups[(0, 10)])
        emb = groups[(0, 0)]
        if all(e.precision == 0 for e in emb):  # fp16 pages: the file's bits
            self.embedding = np.concatenate(
                [np.frombuffer(buf[e.data_offset:e.data_offset + e.data_len].tobytes(), np.float16) for e in emb])
        else:
            self.embedding = raw(emb)
        self.embedding = self.embedding.reshape(self.cfg["vocab"], self.cfg["dim"])
        if cfg.get("tie_word_embeddings"):
            self.lm_head = int4(emb)
        else:
            self.lm_head = int4(groups[(0, 9)])


def host_model(source, overrides: dict | None = None) -> HostModel:
    """The tensors of a `.glacier` model on the host (see HostModel), with the
    same configuration resolution as load_model."""
    gf = source if isinstance(source, GlacierFile) else GlacierFile(source)
    ov = {}
    if gf.path and os.path.exists(gf.path + ".json"):
        with open(gf.path + ".json", "rb") as f:
            ov.update(parse_sidecar(f.read()))
    ov.update(overrides or {})
    return HostModel(gf, resolve_config(gf.geometry(), ov))
