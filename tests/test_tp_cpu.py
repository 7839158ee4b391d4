"""Tensor-parallel decode arithmetic on CPU: gloo ranks replay the sharded step with the oracle.

Each rank holds its TensorParallelShard and runs the reference's cached decode step
(generate.zig:1511-1967, as the oracle's decode_token orders it) on its slice: q/k/v and
gate/up rows, the matching o and down input columns, its own K/V pages.  The o and down
partial products are summed over the ranks with a gloo all-reduce (the step's NCCL
all-reduces on the GPU), and every rank's logits must match the oracle's unsplit decode.

Two splits: by heads (world 2 over 2 kv heads) and by kv-head group and lane (world 4
over 2 kv heads: two ranks share each kv-head group and split its lanes; a rank's
attention output is zero for the lanes it does not attend, as the library's lane split
makes it).  No GPU is needed.
"""
import os
import socket
import sys

import numpy as np
import pytest

import oracle
from helpers import DECODE_LOGIT_TOL, max_err_vs_row_max

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg():
    from glacier_b200.model import ModelConfig
    return ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=500)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_step(sh, cfg, cos, sin, pools, bt, pf_loc, lanes_tok, pos, owned, allreduce):
    """One decode step of this rank's shard for every lane; returns the logits [lanes, vocab]."""
    c = sh.cfg
    D, hd, eps = c["dim"], c["head_dim"], c["eps"]
    Hl, Kl, Fl = c["num_heads"], c["num_kv_heads"], c["hidden"]
    ql, kl = Hl * hd, Kl * hd
    out = []
    for b, tok in enumerate(lanes_tok):
        x = np.asarray(sh.embedding[tok], np.float32).copy()
        for li, L in enumerate(sh.layers):
            h = oracle.rmsnorm(x, L["input_norm"], eps)
            q = oracle.linear_int4(h, *L["wq"], ql, D, 32, bias=L["bq"])[0]
            k = oracle.linear_int4(h, *L["wk"], kl, D, 32, bias=L["bk"])[0]
            v = oracle.linear_int4(h, *L["wv"], kl, D, 32, bias=L["bv"])[0]
            k = oracle.rope_apply(cos, sin, k, pos, Kl, hd)
            oracle.kv_append(pools[b], pf_loc, bt, pos, li, kl, k, v)
            q = oracle.rope_apply(cos, sin, q, pos, Hl, hd)
            if owned(b):
                a = oracle.paged_attention(q, pools[b], pf_loc, bt, pos + 1, li, Hl, Kl, hd)
            else:
                a = np.zeros(ql, np.float32)
            o = allreduce(oracle.linear_int4(a, *L["wo"], D, ql, 32)[0])
            x = x + o
            h2 = oracle.rmsnorm(x, L["post_attn_norm"], eps)
            g = oracle.linear_int4(h2, *L["wg"], Fl, D, 32)[0]
            u = oracle.linear_int4(h2, *L["wu"], Fl, D, 32)[0]
            dn = allreduce(oracle.linear_int4(oracle.silu_mul(g, u), *L["wd"], D, Fl, 32)[0])
            x = x + dn
        hf = oracle.rmsnorm(x, sh.final_norm, eps)
        out.append(oracle.linear_int4(hf, *sh.lm_head, c["vocab"], D, 32)[0])
    return np.stack(out)


def _worker(rank, world, port, lanes, steps, q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "glacier-engine_b200"))
    import torch
    import torch.distributed as dist
    from glacier_b200.model import SyntheticModel, TensorParallelShard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        sh = TensorParallelShard(SyntheticModel(cfg, seed=12), rank, world)

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        c = sh.cfg
        cos, sin = oracle.rope_table(64, c["head_dim"], c["theta"])
        pf_loc = oracle.page_floats(c["num_layers"], c["num_kv_heads"] * c["head_dim"])
        pools = [np.zeros(4 * pf_loc, np.float32) for _ in range(lanes)]
        bt = np.arange(4, dtype=np.int32)
        toks = [(7 * b + 3) % cfg.vocab for b in range(lanes)]
        rec = []
        for pos in range(steps):
            lg = _shard_step(sh, cfg, cos, sin, pools, bt, pf_loc, toks, pos,
                             lambda b: b % sh.lane_groups == sh.lane_index, allreduce)
            rec.append((list(toks), lg))
            toks = [int(np.argmax(lg[b])) for b in range(lanes)]
        q.put((rank, rec))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_shards_decode_like_the_unsplit_oracle(world):
    import torch.multiprocessing as mp
    from glacier_b200.model import SyntheticModel, TensorParallelShard
    cfg = _cfg()
    lanes, steps = 2, 3
    if world == 4:
        s = TensorParallelShard(SyntheticModel(cfg, seed=12, layers=1), 1, 4)
        assert (s.lane_groups, s.lane_index) == (2, 0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, lanes, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    om = oracle.OracleModel(SyntheticModel(cfg, seed=12), rope_positions=64, threads=2)
    pools = [np.zeros(4 * om.page_floats(), np.float32) for _ in range(lanes)]
    bt = np.arange(4, dtype=np.int32)
    for pos in range(steps):
        toks, lg0 = got[0][pos]
        for r in range(1, world):
            assert got[r][pos][0] == toks
            assert max_err_vs_row_max(got[r][pos][1], lg0) <= 1e-6  # every rank ends with the same logits
        for b in range(lanes):
            ol, _ = om.decode_token(pools[b], bt, pos, toks[b])
            assert max_err_vs_row_max(lg0[b], ol) <= DECODE_LOGIT_TOL, (world, b, pos)
