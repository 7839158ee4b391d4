"""Synthetic Qwen2.5-shaped INT4 models and the host side of the decode loop.

The reference runs on converted checkpoints; none is available here, so models
are random-initialised with the BASELINE shapes (the reference does the same for
its own fixtures, src/fixture_gen.zig:18, and tests/model_forward.zig).  Every
INT4 matrix is generated directly in the reference's packing: uniform codes
u in [0, 15] (q = u - 7), one fp16-exact scale of |N(0, 0.02)| magnitude per
32-code group, kept as float32 as the qio payload stores it.

``DeviceModel`` uploads a model through the C ABI; ``DecodeSession`` plays the
host runtime's part (block tables, positions, lanes) around
``glacier_cuda_decode_step`` -- the work the reference's generate.zig /
decode_lane4.zig keep on the host.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib

PAGE_POSITIONS = 16  # src/paged_kv_cache.zig:16


@dataclass(frozen=True)
class ModelConfig:
    num_layers: int
    dim: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    vocab: int
    group: int = 32
    eps: float = 1e-6
    theta: float = 1e6

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    def as_dict(self) -> dict:
        return dict(num_layers=self.num_layers, dim=self.dim, hidden=self.hidden, num_heads=self.num_heads,
                    num_kv_heads=self.num_kv_heads, head_dim=self.head_dim, vocab=self.vocab, group=self.group,
                    eps=self.eps, theta=self.theta)

    def layer_weight_params(self) -> int:
        d, f = self.dim, self.hidden
        return d * self.q_dim + 2 * d * self.kv_dim + self.q_dim * d + 3 * d * f

    def int4_bytes_per_token(self, scale_bytes: int = 2) -> int:
        """Algorithmic weight bytes one decode step streams (codes + scales)."""
        params = self.num_layers * self.layer_weight_params() + self.vocab * self.dim
        return params // 2 + params // self.group * scale_bytes


PRESETS = {
    # BASELINE configs 2, 3 and 4/5 (Qwen2.5 0.5B / 1.5B / 7B shapes).
    "qwen2.5-0.5b": ModelConfig(24, 896, 4864, 14, 2, 64, 151936),
    "qwen2.5-1.5b": ModelConfig(28, 1536, 8960, 12, 2, 128, 151936),
    "qwen2.5-7b": ModelConfig(28, 3584, 18944, 28, 4, 128, 152064),
}


def random_int4(rng: np.random.Generator, out_f: int, in_f: int, group: int = 32):
    """(packed uint8 [out_f*in_f/2], scales float32 [out_f*in_f/group]) with uniform codes."""
    n = out_f * in_f
    packed = rng.integers(0, 256, size=n // 2, dtype=np.uint8)  # two independent uniform codes per byte
    scales = np.abs(rng.standard_normal(n // group, dtype=np.float32) * np.float32(0.02))
    return packed, scales.astype(np.float16).astype(np.float32)


def _random_fp16_table(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """fp16 table built from random bits alone (a 152064 x 3584 table in about a second): random
    sign and 10-bit mantissa, exponent drawn from the four octaves [1/4, 4), so every value is a
    normal fp16 number of magnitude 0.25..4."""
    r = np.frombuffer(rng.bytes(2 * rows * cols), np.uint16).reshape(rows, cols)
    bits = (r & np.uint16(0x83FF)) | ((((r >> np.uint16(10)) & np.uint16(3)) + np.uint16(13)) << np.uint16(10))
    return bits.view(np.float16)


def _fp16_exact(a) -> np.ndarray:
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


class SyntheticModel:
    """Host copy of a random model (what a converted .glacier file would hold)."""

    def __init__(self, cfg: ModelConfig, seed: int = 2024, layers: int | None = None):
        self.config = cfg
        rng = np.random.default_rng(seed)
        nl = cfg.num_layers if layers is None else layers
        c = cfg.as_dict()
        c["num_layers"] = nl
        self.cfg = c
        self.layers = []
        for _ in range(nl):
            L = {
                "wq": random_int4(rng, cfg.q_dim, cfg.dim, cfg.group),
                "wk": random_int4(rng, cfg.kv_dim, cfg.dim, cfg.group),
                "wv": random_int4(rng, cfg.kv_dim, cfg.dim, cfg.group),
                "wo": random_int4(rng, cfg.dim, cfg.q_dim, cfg.group),
                "wg": random_int4(rng, cfg.hidden, cfg.dim, cfg.group),
                "wu": random_int4(rng, cfg.hidden, cfg.dim, cfg.group),
                "wd": random_int4(rng, cfg.dim, cfg.hidden, cfg.group),
                # Qwen2.5 q/k/v biases (forward.zig:51-55).
                "bq": (rng.standard_normal(cfg.q_dim, dtype=np.float32) * np.float32(0.02)),
                "bk": (rng.standard_normal(cfg.kv_dim, dtype=np.float32) * np.float32(0.02)),
                "bv": (rng.standard_normal(cfg.kv_dim, dtype=np.float32) * np.float32(0.02)),
                "input_norm": _fp16_exact(1 + 0.1 * rng.standard_normal(cfg.dim)),
                "post_attn_norm": _fp16_exact(1 + 0.1 * rng.standard_normal(cfg.dim)),
            }
            self.layers.append(L)
        self.embedding = _random_fp16_table(rng, cfg.vocab, cfg.dim)
        self.final_norm = _fp16_exact(1 + 0.1 * rng.standard_normal(cfg.dim))
        self.lm_head = random_int4(rng, cfg.vocab, cfg.dim, cfg.group)


def _rows(w, out_f: int, in_f: int, r0: int, r1: int, group: int = 32):
    """Rows [r0, r1) of an INT4 matrix given as (packed [out_f*in_f/2], scales [out_f*in_f/group])."""
    packed, scales = w
    return (np.ascontiguousarray(packed.reshape(out_f, in_f // 2)[r0:r1]).ravel(),
            np.ascontiguousarray(scales.reshape(out_f, in_f // group)[r0:r1]).ravel())


def _cols(w, out_f: int, in_f: int, c0: int, c1: int, group: int = 32):
    """Input columns [c0, c1) (whole scale groups) of an INT4 matrix."""
    assert c0 % group == 0 and c1 % group == 0
    packed, scales = w
    return (np.ascontiguousarray(packed.reshape(out_f, in_f // 2)[:, c0 // 2:c1 // 2]).ravel(),
            np.ascontiguousarray(scales.reshape(out_f, in_f // group)[:, c0 // group:c1 // group]).ravel())


class TensorParallelShard:
    """Rank `rank`'s share of a model split over `world` GPUs (Megatron split).

    q/k/v rows of this rank's heads (whole GQA groups), gate/up rows of its FFN
    slice, the matching input columns of o and down; norms, biases of its heads,
    embedding and LM head as in the full model.  Its config carries the local
    head counts and FFN width, so the device model is self-consistent; the
    decode step all-reduces the o and down projections over the ranks.

    With more ranks than kv heads (world a multiple of Hkv: 7B at 8 GPUs), each
    kv-head group is shared by lane_groups = world / Hkv ranks: rank r holds
    group r % Hkv's heads and attends the lanes b with b % lane_groups ==
    r // Hkv (lane_index); the FFN is still split over all ranks."""

    def __init__(self, m: SyntheticModel, rank: int, world: int):
        c = dict(m.cfg)
        H, Hkv, hd, F, D, g = c["num_heads"], c["num_kv_heads"], c["head_dim"], c["hidden"], c["dim"], c["group"]
        if Hkv % world == 0:
            heads_split, self.lane_groups, self.lane_index, hr = world, 1, 0, rank
        elif world % Hkv == 0:
            heads_split, self.lane_groups, self.lane_index, hr = Hkv, world // Hkv, rank // Hkv, rank % Hkv
        else:
            heads_split = 0
        # FFN slices in whole blocks of 128 columns where the width gives every rank one (the
        # tensor-core GEMM takes K in multiples of 128), else of one scale group; as even as the
        # blocks allow.
        unit = 128 if F % 128 == 0 and F // 128 >= world else g
        nblk = F // unit if F % unit == 0 else 0
        if not heads_split or H % heads_split or nblk < world or (H // heads_split * hd) % g:
            raise ValueError(f"a {H}/{Hkv}-head, {F}-wide model does not split over {world} GPUs")
        hl, kl = H // heads_split, Hkv // heads_split
        q0, q1 = hr * hl * hd, (hr + 1) * hl * hd
        k0, k1 = hr * kl * hd, (hr + 1) * kl * hd
        f0, f1 = (rank * nblk // world) * unit, ((rank + 1) * nblk // world) * unit
        fl = f1 - f0
        self.ffn_cols = (f0, f1)
        self.cfg = dict(c, num_heads=hl, num_kv_heads=kl, hidden=fl)
        self.config = m.config
        self.rank, self.world = rank, world
        self.layers = []
        for L in m.layers:
            self.layers.append({
                "wq": _rows(L["wq"], H * hd, D, q0, q1, g), "wk": _rows(L["wk"], Hkv * hd, D, k0, k1, g),
                "wv": _rows(L["wv"], Hkv * hd, D, k0, k1, g), "wo": _cols(L["wo"], D, H * hd, q0, q1, g),
                "wg": _rows(L["wg"], F, D, f0, f1, g), "wu": _rows(L["wu"], F, D, f0, f1, g),
                "wd": _cols(L["wd"], D, F, f0, f1, g),
                "bq": L["bq"][q0:q1].copy(), "bk": L["bk"][k0:k1].copy(), "bv": L["bv"][k0:k1].copy(),
                "input_norm": L["input_norm"], "post_attn_norm": L["post_attn_norm"],
            })
        self.embedding, self.final_norm, self.lm_head = m.embedding, m.final_norm, m.lm_head


def tp_unique_id() -> bytes:
    """NCCL unique id for a tensor-parallel group (made on rank 0, handed to every rank)."""
    buf = (C.c_uint8 * 128)()
    _lib.call("glacier_cuda_tp_unique_id", buf)
    return bytes(buf)


def _p(a: np.ndarray):
    return a.ctypes.data


class DeviceModel:
    """A model uploaded to the current CUDA device through the C ABI."""

    def __init__(self, m: SyntheticModel, max_positions: int, scales_f16: bool = True):
        c = m.cfg
        cfgc = _lib.ModelConfigC(c["num_layers"], c["dim"], c["hidden"], c["num_heads"], c["num_kv_heads"],
                                 c["head_dim"], c["vocab"], c["group"], c["eps"], c["theta"], max_positions,
                                 int(scales_f16))
        L = _lib.lib()
        self.cfg = c
        self.max_positions = max_positions
        self.h = _lib.handle(L.glacier_cuda_model_create(C.byref(cfgc)))
        try:
            for i, layer in enumerate(m.layers):
                for key, kind in (("wq", _lib.W_Q), ("wk", _lib.W_K), ("wv", _lib.W_V), ("wo", _lib.W_O),
                                  ("wg", _lib.W_GATE), ("wu", _lib.W_UP), ("wd", _lib.W_DOWN)):
                    self._int4(i, kind, *layer[key])
                for key, kind in (("bq", _lib.B_Q), ("bk", _lib.B_K), ("bv", _lib.B_V),
                                  ("input_norm", _lib.N_INPUT), ("post_attn_norm", _lib.N_POST_ATTN)):
                    a = np.ascontiguousarray(layer[key], np.float32)
                    _lib.call("glacier_cuda_model_load_f32", self.h, i, kind, _p(a), a.size)
            self._int4(-1, _lib.W_LM_HEAD, *m.lm_head)
            fn = np.ascontiguousarray(m.final_norm, np.float32)
            _lib.call("glacier_cuda_model_load_f32", self.h, -1, _lib.N_FINAL, _p(fn), fn.size)
            if np.asarray(m.embedding).dtype == np.float32:
                # f32 rows (a model file's INT4, bf16 or fp32 embedding): kept as they are.
                emb32 = np.ascontiguousarray(m.embedding, np.float32)
                _lib.call("glacier_cuda_model_load_embedding_f32", self.h, _p(emb32), emb32.size)
            else:
                emb = np.ascontiguousarray(m.embedding, np.float16).view(np.uint16)
                _lib.call("glacier_cuda_model_load_embedding_f16", self.h, _p(emb), emb.size)
            _lib.call("glacier_cuda_model_finalize", self.h)
        except Exception:
            self.close()
            raise

    @classmethod
    def from_glacier(cls, gf, cfg: dict, max_positions: int, scales_f16: bool = True) -> "DeviceModel":
        """Loads an admitted GlacierFile with a resolved config (see glacier_file.load_model)."""
        self = cls.__new__(cls)
        cfgc = _lib.ModelConfigC(cfg["num_layers"], cfg["dim"], cfg["hidden"], cfg["num_heads"],
                                 cfg["num_kv_heads"], cfg["head_dim"], cfg["vocab"], cfg["group"], cfg["eps"],
                                 cfg["theta"], max_positions, int(scales_f16))
        self.cfg = {k: cfg[k] for k in ("num_layers", "dim", "hidden", "num_heads", "num_kv_heads", "head_dim",
                                        "vocab", "group", "eps", "theta")}
        self.max_positions = max_positions
        self.h = _lib.handle(_lib.lib().glacier_cuda_model_create(C.byref(cfgc)))
        try:
            _lib.call("glacier_cuda_model_load_glacier", self.h, gf._ptr, gf.size,
                      int(cfg.get("tie_word_embeddings", False)))
            _lib.call("glacier_cuda_model_finalize", self.h)
        except Exception:
            self.close()
            raise
        return self

    @classmethod
    def from_runtime_image(cls, img, max_positions: int, scales_f16: bool = True) -> "DeviceModel":
        """Loads an admitted RuntimeImage with the config its header carries (see runtime_image.load_model)."""
        info = img.model_info()
        cfg = dict(num_layers=info.num_layers, dim=info.dim, hidden=info.hidden, num_heads=info.num_heads,
                   num_kv_heads=info.num_kv_heads, head_dim=info.head_dim, vocab=info.vocab,
                   group=info.group_size, eps=info.rms_eps, theta=info.rope_theta)
        self = cls.__new__(cls)
        cfgc = _lib.ModelConfigC(cfg["num_layers"], cfg["dim"], cfg["hidden"], cfg["num_heads"],
                                 cfg["num_kv_heads"], cfg["head_dim"], cfg["vocab"], cfg["group"], cfg["eps"],
                                 cfg["theta"], max_positions, int(scales_f16))
        self.cfg = cfg
        self.max_positions = max_positions
        self.h = _lib.handle(_lib.lib().glacier_cuda_model_create(C.byref(cfgc)))
        try:
            _lib.call("glacier_cuda_model_load_glrt", self.h, img._ptr, img.size, C.byref(img.options))
            _lib.call("glacier_cuda_model_finalize", self.h)
        except Exception:
            self.close()
            raise
        return self

    def enable_tensor_parallel(self, rank: int, world: int, unique_id: bytes, lane_groups: int = 1,
                               lane_index: int = 0):
        """Joins the tensor-parallel group (blocks until every rank has joined); with
        lane_groups > 1 this rank attends the lanes b with b % lane_groups == lane_index
        (TensorParallelShard gives both)."""
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        _lib.call("glacier_cuda_model_tp_init", self.h, rank, world, buf)
        if lane_groups > 1:
            _lib.call("glacier_cuda_model_tp_lanes", self.h, lane_groups, lane_index)

    def _int4(self, layer, kind, packed, scales):
        packed = np.ascontiguousarray(packed, np.uint8)
        scales = np.ascontiguousarray(scales, np.float32)
        _lib.call("glacier_cuda_model_load_int4", self.h, layer, kind, _p(packed), packed.size, _p(scales),
                  scales.size)

    def close(self):
        if getattr(self, "h", None):
            _lib.lib().glacier_cuda_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: ctypes / module globals may already be gone
            pass


class DecodeSession:
    """Host-side lane bookkeeping around glacier_cuda_decode_step.

    Lane b owns pages [b*max_pages, (b+1)*max_pages) of one KV pool (the
    reference's per-request page table, paged_kv_cache.zig:44-48); torch only
    provides device memory and the stream.
    """

    def __init__(self, dm: DeviceModel, lanes: int, max_pages: int, reserve_lanes: int | None = None):
        import torch
        self.torch = torch
        self.dm, self.lanes, self.max_pages = dm, lanes, max_pages
        L = _lib.lib()
        _lib.call("glacier_cuda_model_reserve", dm.h, reserve_lanes or lanes, max_pages)
        self.kv = _lib.handle(L.glacier_cuda_kv_create(dm.h, lanes * max_pages))
        self.page_floats = L.glacier_cuda_kv_page_floats(self.kv)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.block_tables = torch.arange(lanes * max_pages, dtype=torch.int32, device=dev).reshape(lanes, max_pages)
        self.tokens = torch.zeros(lanes, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(lanes, dtype=torch.int32, device=dev)
        self.out = torch.zeros(lanes, dtype=torch.int32, device=dev)
        self.status = torch.zeros(lanes, dtype=torch.int32, device=dev)

    def pages(self):
        """The KV pool as a torch view [num_pages, page_floats] (device memory of the library)."""
        ptr = _lib.lib().glacier_cuda_kv_pages(self.kv)
        n = self.lanes * self.max_pages * self.page_floats
        return _ptr_tensor(self.torch, ptr, n).view(self.lanes * self.max_pages, self.page_floats)

    def step(self, tokens=None, positions=None, eligible=None, logits=None, stream=None):
        """One decode step on device tensors already in self.tokens / self.positions."""
        torch = self.torch
        if tokens is not None:
            self.tokens.copy_(torch.as_tensor(tokens, dtype=torch.int32))
        if positions is not None:
            self.positions.copy_(torch.as_tensor(positions, dtype=torch.int32))
        s = stream if stream is not None else torch.cuda.current_stream()
        words = 0 if eligible is None else eligible.shape[-1]
        _lib.call("glacier_cuda_decode_step", self.dm.h, self.kv, self.lanes, self.tokens.data_ptr(),
                  self.positions.data_ptr(), self.block_tables.data_ptr(), self.max_pages,
                  None if eligible is None else eligible.data_ptr(), words, self.out.data_ptr(),
                  self.status.data_ptr(), None if logits is None else logits.data_ptr(), s.cuda_stream)
        return self.out

    def capture_greedy_step(self, stream=None):
        """Records one greedy continuation step as a CUDA graph: decode_step on self.tokens and
        self.positions, then tokens <- the new token ids and positions += 1.  replay_greedy_step()
        runs it again; all of its inputs live in device memory, so a replay is the same step as a
        fresh launch sequence, minus the host launch work and inter-launch gaps."""
        torch = self.torch
        s = stream if stream is not None else torch.cuda.current_stream()
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph, stream=s):
            out = self.step(stream=s)
            self.tokens.copy_(out)
            self.positions.add_(1)
        return self._graph

    def replay_greedy_step(self):
        """One replay of the graph recorded by capture_greedy_step (on its capture stream)."""
        self._graph.replay()
        return self.out

    def prefill(self, prompt, lane: int = 0, start: int = 0, eligible=None, logits=None, stream=None):
        """Feeds prompt tokens (host sequence or device int32 tensor) of one request at positions
        start.. through lane `lane`'s block table; returns the device int32 tensor [1] holding
        the greedy token that follows (generate.zig prompt loop, batched)."""
        torch = self.torch
        dev = self.tokens.device
        toks = torch.as_tensor(prompt, dtype=torch.int32).to(dev).contiguous()
        out = torch.empty(1, dtype=torch.int32, device=dev)
        status = torch.empty(1, dtype=torch.int32, device=dev)
        s = stream if stream is not None else torch.cuda.current_stream()
        words = 0 if eligible is None else eligible.shape[-1]
        _lib.call("glacier_cuda_prefill", self.dm.h, self.kv, toks.data_ptr(), toks.numel(), start,
                  self.block_tables[lane].data_ptr(), self.max_pages,
                  None if eligible is None else eligible.data_ptr(), words, out.data_ptr(), status.data_ptr(),
                  None if logits is None else logits.data_ptr(), s.cuda_stream)
        self.last_status = status
        return out

    def close(self):
        self._graph = None  # a recorded step references this session's buffers
        if getattr(self, "kv", None):
            _lib.lib().glacier_cuda_kv_destroy(self.kv)
            self.kv = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: ctypes / module globals may already be gone
            pass


def _ptr_tensor(torch, ptr: int, numel: int):
    """A float32 torch view of library-owned device memory (no copy, no ownership)."""

    class _Holder:
        pass

    h = _Holder()
    h.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                  "strides": None}
    return torch.as_tensor(h, device="cuda")
