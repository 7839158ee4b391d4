"""Host logic of the multi-GPU bench on CPU: gloo ranks, world size 2.

The decode path partitions lanes across GPUs with no data-path collective; the
only cross-rank steps are the barrier and the max-over-ranks of the timed
region.  These run here on the gloo backend.
"""
import os
import socket
import sys
import types

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ws, r, local = bench.dist_setup()
    args = types.SimpleNamespace(seed=2024, ctx_min=256, ctx_max=4096)
    ctx = bench.lane_contexts(args, 64, r)
    # rank-dependent timings: the reported job time is the slowest rank's
    t = bench.max_over_ranks([1.0 + r, 10.0 - r], ws, "cpu")
    dist.barrier()
    out[rank] = (ws, r, local, ctx.tolist(), t)
    dist.destroy_process_group()


def test_two_rank_lane_partition_and_max_timing():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    r0, r1 = out[0], out[1]
    assert (r0[0], r0[1], r0[2]) == (2, 0, 0) and (r1[0], r1[1], r1[2]) == (2, 1, 1)
    # each rank decodes its own 64 lanes with its own contexts, in the configured range
    c0, c1 = np.array(r0[3]), np.array(r1[3])
    assert c0.shape == c1.shape == (64,) and not np.array_equal(c0, c1)
    assert c0.min() >= 256 and c1.max() <= 4096
    # both ranks agree on the element-wise maximum
    assert r0[4] == r1[4] == [2.0, 10.0]


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    args = types.SimpleNamespace(model="qwen2.5-7b", seed=1, layers=1, lanes=2, warmup=1, steps=1, gpus=2)
    assert bench.run_reference(args) is None
    assert capsys.readouterr().out == ""
