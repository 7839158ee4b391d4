"""The prepared runtime image (`.glrt`) through the C ABI.

``RuntimeImage`` admits an image as the reference's
``MappedImage.openWithOptions`` does (src/model/runtime_image.zig:805-850);
``load_model`` builds a device-resident model from it as
``loader.loadPreparedWithOptions`` does (src/loader.zig:200-385).  Parsing,
checksums, digests and the layout transforms all run in the library
(csrc/runtime_image.cu).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from .glacier_file import _map_file

ENCODINGS = {0: "raw_f32", 1: "int4", 2: "pair_nibble"}
PACKED_LAYOUTS = {0: "row_major", 1: "rows4_k16", 0xFFFF: "none"}
ROLES = {0: "tensor", 1: "mlp_gate_up_pair"}
STREAMS = ("packed_weights", "scales_f32", "scales_f16", "scales_f16_rows4", "raw")
GLOBAL_LAYER = 0xFFFFFFFF


class RuntimeImage:
    """An admitted `.glrt` image held in host memory."""

    def __init__(self, source, verify_crc: bool = True, verify_digest: bool = True, allow_v1: bool = True,
                 abi_policy: str | None = None, expected_source_fingerprint: bytes | None = None):
        if isinstance(source, (str, os.PathLike)):
            self._buf = _map_file(os.fspath(source))
        else:
            self._buf = np.frombuffer(memoryview(source), np.uint8)
        self._fp = None
        if expected_source_fingerprint is not None:
            if len(expected_source_fingerprint) != 32:
                raise ValueError("a source fingerprint is 32 bytes")
            self._fp = np.frombuffer(bytes(expected_source_fingerprint), np.uint8).copy()
        policy = {None: 0, "portable": 1, "aarch64": 2}[abi_policy]
        self.options = _lib.GlrtOptions(int(not verify_crc), int(not verify_digest), int(not allow_v1), policy,
                                        self._fp.ctypes.data if self._fp is not None else None)
        self.info = _lib.GlrtInfo()
        _lib.call("glacier_cuda_glrt_open", self._ptr, self.size, C.byref(self.options), C.byref(self.info))

    @property
    def _ptr(self):
        return self._buf.ctypes.data if self._buf.size else None

    @property
    def size(self) -> int:
        return int(self._buf.size)

    @property
    def num_records(self) -> int:
        return int(self.info.record_count)

    def record(self, index: int) -> _lib.GlrtEntry:
        e = _lib.GlrtEntry()
        _lib.call("glacier_cuda_glrt_record", self._ptr, self.size, index, C.byref(e))
        return e

    def records(self) -> list[_lib.GlrtEntry]:
        """Every record, from one structural admission of the image."""
        n = self.num_records
        arr = (_lib.GlrtEntry * max(n, 1))()
        count = C.c_uint64()
        _lib.call("glacier_cuda_glrt_records", self._ptr, self.size, arr, n, C.byref(count))
        return list(arr[:count.value])

    def stream(self, rec: _lib.GlrtEntry, name: str) -> np.ndarray:
        """The bytes of one stream of a record (a view into the image)."""
        s = STREAMS.index(name)
        off, n = rec.stream_offset[s], rec.stream_len[s]
        return self._buf[off:off + n]

    def model_info(self) -> _lib.GlrtInfo:
        """Header config plus the prepared-model schema checks: MLP form and INT4 group."""
        info = _lib.GlrtInfo()
        _lib.call("glacier_cuda_glrt_model_info", self._ptr, self.size, C.byref(self.options), C.byref(info))
        return info


def load_model(source, max_positions: int, scales_f16: bool = True, **open_options):
    """A finalized DeviceModel built from a `.glrt` image on the current device."""
    from .model import DeviceModel
    img = source if isinstance(source, RuntimeImage) else RuntimeImage(source, **open_options)
    return DeviceModel.from_runtime_image(img, max_positions, scales_f16)


def rows4_k16_to_row_major(packed: np.ndarray, out_f: int, in_f: int) -> np.ndarray:
    src = np.ascontiguousarray(packed, np.uint8)
    dst = np.empty(out_f * in_f // 2, np.uint8)
    _lib.call("glacier_cuda_rows4_k16_to_row_major", src.ctypes.data, dst.ctypes.data, out_f, in_f)
    return dst


def rows4_scales_to_row_major(scales_f16: np.ndarray, out_f: int, groups_per_row: int) -> np.ndarray:
    src = np.ascontiguousarray(scales_f16, np.float16).view(np.uint16)
    dst = np.empty(out_f * groups_per_row, np.float32)
    _lib.call("glacier_cuda_rows4_scales_to_row_major", src.ctypes.data, dst.ctypes.data, out_f, groups_per_row)
    return dst


def pair_nibble_split(pairs: np.ndarray, pair_scales_f16: np.ndarray, out_f: int, in_f: int, group: int):
    """(gate packed, up packed, gate scales f32, up scales f32), all row-major."""
    p = np.ascontiguousarray(pairs, np.uint8)
    s = np.ascontiguousarray(pair_scales_f16, np.float16).view(np.uint16)
    gate = np.empty(out_f * in_f // 2, np.uint8)
    up = np.empty_like(gate)
    gs = np.empty(out_f * in_f // group, np.float32)
    us = np.empty_like(gs)
    _lib.call("glacier_cuda_pair_nibble_split", p.ctypes.data, s.ctypes.data, out_f, in_f, group, gate.ctypes.data,
              up.ctypes.data, gs.ctypes.data, us.ctypes.data)
    return gate, up, gs, us


class HostModel:
    """A prepared image's tensors as host arrays in glacier_b200.model's layout
    (INT4 as row-major (packed, f32 scales), norms and biases as f32), put back
    from rows4_k16 / rows4-grid / PairNibble form by the library's layout
    transforms exactly as its loader does, so TensorParallelShard can cut a
    prepared image into per-GPU shards.  The embedding becomes f32 rows
    (dequantizeRow: code offset times the f32 group scale)."""

    KINDS = {1: "wq", 2: "wk", 3: "wv", 4: "wo", 5: "wu", 6: "wd", 7: "wg", 8: "input_norm", 11: "post_attn_norm",
             12: "bq", 13: "bk", 14: "bv"}

    def __init__(self, img: RuntimeImage):
        from .model import ModelConfig
        i = img.model_info()
        if i.group_size == 0:
            raise ValueError("the image holds no INT4 records")
        self.cfg = dict(num_layers=i.num_layers, dim=i.dim, hidden=i.hidden, num_heads=i.num_heads,
                        num_kv_heads=i.num_kv_heads, head_dim=i.head_dim, vocab=i.vocab, group=i.group_size,
                        eps=i.rms_eps, theta=i.rope_theta)
        self.config = ModelConfig(**self.cfg)
        recs = img.records()

        def int4(r):
            n = r.out_f * r.in_f
            pk = img.stream(r, "packed_weights")
            packed = np.array(pk) if r.packed_layout == 0 else rows4_k16_to_row_major(pk, r.out_f, r.in_f)
            if img.stream(r, "scales_f32").size:
                scales = np.frombuffer(img.stream(r, "scales_f32").tobytes(), np.float32).copy()
            elif img.stream(r, "scales_f16").size:
                scales = np.frombuffer(img.stream(r, "scales_f16").tobytes(), np.float16).astype(np.float32)
            else:
                grid = np.frombuffer(img.stream(r, "scales_f16_rows4").tobytes(), np.float16)
                scales = rows4_scales_to_row_major(grid, r.out_f, r.in_f // r.group_size)
            assert packed.size == -(-n // 2)
            return packed, scales

        def raw(r):
            return np.frombuffer(img.stream(r, "raw").tobytes(), np.float32).copy()

        self.layers = [dict(bq=None, bk=None, bv=None) for _ in range(i.num_layers)]
        self.lm_head = None
        self.final_norm = None
        emb = None
        for r in recs:
            if r.layer_idx != GLOBAL_LAYER and not 0 <= r.layer_idx < i.num_layers:
                raise ValueError(f"record of layer {r.layer_idx} in an image of {i.num_layers} layers")
            if r.role == 1:  # PairNibble gate/up
                grid = np.frombuffer(img.stream(r, "scales_f16_rows4").tobytes(), np.float16)
                g, u, gs, us = pair_nibble_split(img.stream(r, "packed_weights"), grid, r.out_f, r.in_f,
                                                 r.group_size)
                self.layers[r.layer_idx]["wg"], self.layers[r.layer_idx]["wu"] = (g, gs), (u, us)
            elif r.layer_idx == GLOBAL_LAYER:
                if r.tensor_kind == 10:
                    self.final_norm = raw(r)
                elif r.tensor_kind == 0:
                    emb = int4(r)
                elif r.tensor_kind == 9:
                    self.lm_head = int4(r)
            else:
                name = self.KINDS.get(r.tensor_kind)
                if name is None:
                    raise ValueError(f"record kind {r.tensor_kind} is not part of this decode path")
                self.layers[r.layer_idx][name] = int4(r) if name.startswith("w") else raw(r)
        for n, L in enumerate(self.layers):
            for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "input_norm", "post_attn_norm"):
                if name not in L:
                    raise ValueError(f"layer {n} has no {name}")
        if emb is None:
            raise ValueError("the image has no embedding record")
        if getattr(self, "final_norm", None) is None:
            raise ValueError("the image has no final norm record")
        if self.lm_head is None and not i.tie_embeddings:
            raise ValueError("the image has no LM head record and does not tie it to the embedding")
        packed, scales = emb
        q = np.stack([packed & 15, packed >> 4], -1).reshape(-1)[: i.vocab * i.dim].astype(np.float32) - 7
        self.embedding = (q * np.repeat(scales, i.group_size)[: q.size]).reshape(i.vocab, i.dim)
        if i.tie_embeddings:
            self.lm_head = emb


def host_model(source, **open_options) -> HostModel:
    """The tensors of a `.glrt` image on the host (see HostModel)."""
    img = source if isinstance(source, RuntimeImage) else RuntimeImage(source, **open_options)
    return HostModel(img)
