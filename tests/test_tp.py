"""Tensor parallelism (Megatron split) over GPUs.

On CPU: the shard arithmetic, checked with the oracle.  q/k/v and gate/up rows
of the shards concatenate to the full matrices, and the row-parallel o and down
projections summed over the ranks give the full projection.

On 2+ GPUs: a TP=2 decode, one process per GPU over NCCL, against the oracle.
"""
import os
import socket
import sys

import numpy as np
import pytest

import oracle
from helpers import DECODE_LOGIT_TOL, REL_TOL, max_err_vs_row_max, max_rel_err

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(kind="small"):
    from glacier_b200.model import ModelConfig
    if kind == "7b-heads":  # the 7B head layout (28 / 4 heads of 128): 8 ranks share 4 kv-head groups
        return ModelConfig(num_layers=2, dim=512, hidden=2048, num_heads=28, num_kv_heads=4, head_dim=128,
                           vocab=1000)
    return ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)


def test_tp_shards_reassemble_the_projections():
    from glacier_b200.model import SyntheticModel, TensorParallelShard
    cfg = _cfg()
    m = SyntheticModel(cfg, seed=3)
    world = 2
    shards = [TensorParallelShard(m, r, world) for r in range(world)]
    L = m.layers[0]
    rng = np.random.default_rng(0)
    # row-parallel: q and gate outputs concatenate
    x = rng.standard_normal(cfg.dim, dtype=np.float32)
    full_q = oracle.linear_int4(x, *L["wq"], cfg.q_dim, cfg.dim, 32)
    parts = [oracle.linear_int4(x, *s.layers[0]["wq"], cfg.q_dim // world, cfg.dim, 32) for s in shards]
    assert np.array_equal(np.concatenate(parts, axis=-1), full_q)
    full_g = oracle.linear_int4(x, *L["wg"], cfg.hidden, cfg.dim, 32)
    parts = [oracle.linear_int4(x, *s.layers[0]["wg"], cfg.hidden // world, cfg.dim, 32) for s in shards]
    assert np.array_equal(np.concatenate(parts, axis=-1), full_g)
    # column-parallel o and down: the ranks' partial products sum to the full projection
    a = rng.standard_normal(cfg.q_dim, dtype=np.float32)
    full_o = oracle.linear_int4(a, *L["wo"], cfg.dim, cfg.q_dim, 32)
    ql = cfg.q_dim // world
    part = sum(oracle.linear_int4(a[r * ql:(r + 1) * ql], *shards[r].layers[0]["wo"], cfg.dim, ql, 32)
               for r in range(world))
    assert max_rel_err(part, full_o) <= REL_TOL
    h = rng.standard_normal(cfg.hidden, dtype=np.float32)
    full_d = oracle.linear_int4(h, *L["wd"], cfg.dim, cfg.hidden, 32)
    fl = cfg.hidden // world
    part = sum(oracle.linear_int4(h[r * fl:(r + 1) * fl], *shards[r].layers[0]["wd"], cfg.dim, fl, 32)
               for r in range(world))
    assert max_rel_err(part, full_d) <= REL_TOL
    assert shards[1].cfg["num_heads"] == 4 and shards[1].cfg["num_kv_heads"] == 1 and shards[1].cfg["hidden"] == 256


def test_tp_rejects_uneven_splits():
    from glacier_b200.model import SyntheticModel, TensorParallelShard
    m = SyntheticModel(_cfg(), seed=1)
    with pytest.raises(ValueError):
        TensorParallelShard(m, 0, 3)  # 3 GPUs neither divide 2 kv heads nor a multiple of them
    s = TensorParallelShard(m, 3, 4)  # 4 GPUs over 2 kv heads: two ranks per kv-head group
    assert (s.lane_groups, s.lane_index) == (2, 1)
    assert s.cfg["num_heads"] == 4 and s.cfg["num_kv_heads"] == 1 and s.cfg["hidden"] == 128


def test_tp_ffn_slices_are_whole_128_column_blocks():
    """7B's FFN (18944 = 148 x 128) over 8 ranks: 18 or 19 blocks of 128 each, so every local
    down projection keeps K a multiple of 128 (the tensor-core GEMM's chunk); the slices tile F."""
    from glacier_b200.model import ModelConfig, SyntheticModel, TensorParallelShard
    cfg = ModelConfig(num_layers=1, dim=64, hidden=18944, num_heads=28, num_kv_heads=4, head_dim=128, vocab=64)
    m = SyntheticModel(cfg, seed=2)
    for world in (2, 4, 8):
        cols = [TensorParallelShard(m, r, world).ffn_cols for r in range(world)]
        assert cols[0][0] == 0 and cols[-1][1] == cfg.hidden
        assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
        assert all((f1 - f0) % 128 == 0 and f1 > f0 for f0, f1 in cols)
        assert max(f1 - f0 for f0, f1 in cols) - min(f1 - f0 for f0, f1 in cols) <= 128


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, lanes, prompt_len, new_tokens, out, kind):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "glacier-engine_b200"))
    import torch
    import torch.distributed as dist
    from glacier_b200.model import DecodeSession, DeviceModel, SyntheticModel, TensorParallelShard, tp_unique_id
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = _cfg(kind)
    m = SyntheticModel(cfg, seed=5)
    max_pages = -(-(prompt_len + new_tokens) // 16)
    shard = TensorParallelShard(m, rank, world)
    dm = DeviceModel(shard, max_positions=max_pages * 16)
    uid = [tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    dm.enable_tensor_parallel(rank, world, uid[0], shard.lane_groups, shard.lane_index)
    sess = DecodeSession(dm, lanes, max_pages, reserve_lanes=max(lanes, 8))
    rng = np.random.default_rng(9)
    prompts = rng.integers(0, cfg.vocab, size=(lanes, prompt_len)).astype(np.int32)
    logits = torch.empty((lanes, cfg.vocab), device="cuda")
    rec = []
    cur = prompts[:, 0].copy()
    for pos in range(prompt_len + new_tokens - 1):
        tok = sess.step(tokens=cur, positions=[pos] * lanes, logits=logits).cpu().numpy()
        rec.append((cur.copy(), tok.copy(), logits.cpu().numpy().copy()))
        cur = prompts[:, pos + 1].copy() if pos + 1 < prompt_len else tok.astype(np.int32)
    out[rank] = rec
    sess.close()
    dm.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world,kind", [(2, "small"), (4, "small"), (8, "7b-heads")])
def test_tp_decode_matches_oracle(world, kind):
    """TP decode over `world` GPUs vs the oracle: a head split at 2 GPUs; at 4 GPUs on 2 kv heads
    and at 8 GPUs on the 7B head layout (4 kv heads), two ranks share each kv-head group and
    split its lanes."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"tensor parallelism over {world} GPUs needs {world} GPUs")
    import torch.multiprocessing as mp
    from glacier_b200.model import SyntheticModel
    lanes, prompt_len, new_tokens = 8, 6, 4  # 8 lanes: tensor-core projections
    out = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_tp_worker, args=(world, _free_port(), lanes, prompt_len, new_tokens, out, kind),
                       nprocs=world, start_method="spawn", join=True)
    r0 = out[0]
    for r in range(1, world):
        for (_, ta, _), (_, tb, _) in zip(r0, out[r]):
            assert np.array_equal(ta, tb)  # every rank produces the same tokens
    r1 = out[1]
    cfg = _cfg(kind)
    m = SyntheticModel(cfg, seed=5)
    max_pages = -(-(prompt_len + new_tokens) // 16)
    om = oracle.OracleModel(m, rope_positions=max_pages * 16, threads=4)
    pools = [np.zeros(max_pages * om.page_floats(), np.float32) for _ in range(lanes)]
    bt = np.arange(max_pages, dtype=np.int32)
    live = [True] * lanes
    for pos, ((cur, tok0, lg0), (_, tok1, lg1)) in enumerate(zip(r0, r1)):
        assert np.array_equal(tok0, tok1)  # every rank produces the same tokens
        for b in range(lanes):
            ol, _ = om.decode_token(pools[b], bt, pos, int(cur[b]))
            if not live[b]:
                continue
            assert max_err_vs_row_max(lg0[b], ol) <= DECODE_LOGIT_TOL, (b, pos)
            if pos >= prompt_len - 1 and tok0[b] != oracle.argmax(ol):
                top2 = np.sort(ol)[-2:]
                assert (top2[1] - top2[0]) < 1e-3 * max(1.0, abs(float(top2[1])))
                live[b] = False
