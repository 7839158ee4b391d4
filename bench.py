"""Benchmark: INT4 decode of the Qwen2.5-7B-shaped synthetic model on B200.

Workload (the metric's 7B shape at batch 64): 64 decode
lanes per GPU, contexts drawn uniformly from [256, 4096], greedy decoding.  One
step = one decode step of every lane (64 new tokens per GPU).  Weights are
random-initialised in the reference's INT4 g32 packing (no checkpoint exists
here); KV pages are pre-filled with random values (FP32, the reference's KV
format) so that each lane starts at its drawn context length.  The working set
(4.0 GB of weights + KV) is far larger than the 126 MB L2, so no flush is
needed between steps.

  python bench.py [--gpus N --steps K --warmup W]          this implementation
  python bench.py --impl reference [...]                     the reference's CPU
                                                             path (C oracle port)
Multi-GPU: one process per GPU (torchrun); lanes are partitioned by GPU with a
full weight replica each and no collective on the data path (weak scaling).
Rank 0 prints one JSON line.

Beside the headline, the same line carries the other BASELINE configurations,
each with its own roofline and CPU baseline: on one GPU `gemv_config1` (the
4864 x 896 GEMV), `config2` (0.5B, batch 1, 128 tokens after a 512-token
prefill), `config3` (1.5B, 8 lanes, 256 tokens each), `prefill` (7B prompts of
128 / 512 / 2048 tokens) and `batch1` (7B, one lane); under torchrun
`strong_scaling` (64 lanes in total split over the N GPUs) and `tp` (one
64-lane job over N tensor-parallel GPUs, where the 7B heads divide by N).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "glacier-engine_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "INT4 decode tok/s and achieved HBM GB/s (Qwen2.5-7B shape, batch 1 and 64)"
UNIT = "tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["glacier", "reference"], default="glacier")
    ap.add_argument("--lanes", type=int, default=64)
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--model-file", default=None,
                    help="run on the tensors of a .glacier file or .glrt image instead of the preset's synthetic model")
    ap.add_argument("--ctx-min", type=int, default=256)
    ap.add_argument("--ctx-max", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the timed CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="build only this many decoder layers (small cases for ncu captures; not a bench number)")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel degree: with --tp N under torchrun (N ranks) the ranks share one model "
                         "and one set of lanes (strong scaling); default 1 = lane partition (weak scaling)")
    ap.add_argument("--workload", choices=["decode", "prefill"], default="decode",
                    help="decode: the headline 64-lane step; prefill: one prompt of --tokens tokens (config 4)")
    ap.add_argument("--tokens", type=int, default=2048, help="prompt length for --workload prefill")
    ap.add_argument("--profile-steps", type=int, default=10,
                    help="decode steps of the per-kernel-class event pass that follows the timed region")
    ap.add_argument("--no-extras", action="store_true",
                    help="headline only: skip the other configurations' keys (small cases for profiling)")
    a = ap.parse_args()
    if a.model_file and a.layers is not None:
        ap.error("--layers cuts the synthetic preset; it does not apply to --model-file")
    return a


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms from before the
    warm-up until after the timed region; summary() keeps the samples that arrived
    inside the timed window (host timestamps taken with the device synchronised)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, interval_ms: int = 50):
        self.index = index
        self.interval_ms = interval_ms
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def start_window(self):
        self.t0 = time.perf_counter()

    def end_window(self):
        self.t1 = time.perf_counter()

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(2 * self.interval_ms / 1e3)  # let the sample after the window arrive
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lo = self.t0 if self.t0 is not None else -1e18
        hi = (self.t1 if self.t1 is not None else 1e18) + self.interval_ms / 1e3
        for ts, ln in self.lines:
            if not (lo <= ts <= hi):
                continue
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def lane_contexts(args, lanes: int, rank: int) -> np.ndarray:
    """Contexts of a rank's lanes: one seeded draw from U[ctx_min, ctx_max], the same multiset on
    every rank (in a rank-specific order), so that per-GPU KV bytes -- and with them per-GPU work
    -- stay fixed as the lane partition grows (independent draws per rank differ by about 10% in
    total context at 64 lanes, and the slowest rank sets the job's time)."""
    ctx = np.random.default_rng(args.seed).integers(args.ctx_min, args.ctx_max + 1, size=lanes)
    if rank:
        ctx = np.random.default_rng(args.seed + 1000 * rank).permutation(ctx)
    return ctx.astype(np.int32)


def max_over_ranks(values, world_size: int, device) -> list:
    """Element-wise maximum of per-rank timings (the job is as slow as its slowest rank)."""
    if world_size <= 1:
        return [float(v) for v in values]
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def pin_cores(local: int, local_world: int) -> int:
    """Under torchrun, gives each rank its own slice of the host cores (so the ranks' launch
    threads do not compete); returns the cores this process may use."""
    try:
        cpus = sorted(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
    if local_world > 1 and len(cpus) >= local_world:
        per = len(cpus) // local_world
        mine = cpus[local * per:(local + 1) * per]
        os.sched_setaffinity(0, mine)
        return len(mine)
    return len(cpus)


def cpu_threads() -> int:
    try:
        return max(1, min(16, len(os.sched_getaffinity(0))))
    except AttributeError:
        return max(1, min(16, os.cpu_count() or 1))


def time_cpu_oracle(model, ctxs, args, budget_s: float, max_tokens: int | None = None) -> dict:
    """Greedy decode on the C oracle (the reference's portable FP32 path restated),
    one lane at a time at its drawn context, with the reference's row-split
    threading over all host cores.  Returns tokens/s over the sample."""
    import oracle
    threads = cpu_threads()
    c = model.cfg
    kv_dim = c["num_kv_heads"] * c["head_dim"]
    om = oracle.OracleModel(model, rope_positions=int(max(ctxs)) + 64, threads=threads)
    pf = om.page_floats()
    rng = np.random.default_rng(args.seed + 7)
    tokens = 0
    t_total = 0.0
    lane = 0
    while True:
        ctx = int(ctxs[lane % len(ctxs)])
        pages = -(-(ctx + 1) // 16)
        pool = rng.standard_normal(pages * pf, dtype=np.float32)
        bt = np.arange(pages, dtype=np.int32)
        tok = int(rng.integers(0, c["vocab"]))
        t0 = time.perf_counter()
        logits, _ = om.decode_token(pool, bt, ctx, tok)
        oracle.argmax(logits)
        t_total += time.perf_counter() - t0
        tokens += 1
        lane += 1
        if (max_tokens is not None and tokens >= max_tokens) or (max_tokens is None and t_total >= budget_s):
            break
    return {"value": tokens / t_total, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{tokens} greedy tokens of single lanes at their drawn contexts "
                      f"(mean ctx {int(np.mean(ctxs[:max(1, min(tokens, len(ctxs)))]))}), full "
                      f"{c['num_layers']}-layer model + LM head, {kv_dim}-float KV rows",
            "seconds": t_total}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------

def bench_model(args):
    """(ModelConfig, host model) the bench runs: the preset's synthetic model with
    random weights, or the tensors of --model-file (a .glacier file or a .glrt
    image, read through the library's own readers)."""
    from glacier_b200.model import PRESETS, SyntheticModel
    if getattr(args, "model_file", None):
        if args.model_file.endswith(".glrt"):
            from glacier_b200.runtime_image import host_model
        else:
            from glacier_b200.glacier_file import host_model
        m = host_model(args.model_file)
        return m.config, m
    cfg = PRESETS[args.model]
    return cfg, SyntheticModel(cfg, seed=args.seed, layers=args.layers)


def data_label(args) -> str:
    return f"model file {os.path.basename(args.model_file)}" if getattr(args, "model_file", None) else "synthetic"


def model_label(args, cfg, layers: int | None = None) -> str:
    """The model a line measures: the preset's name, or the model file's name with the
    geometry read from it."""
    nl = layers if layers is not None else cfg.num_layers
    if getattr(args, "model_file", None):
        return (f"{os.path.basename(args.model_file)} ({nl} layers, dim {cfg.dim}, ffn {cfg.hidden}, "
                f"{cfg.num_heads}/{cfg.num_kv_heads} heads of {cfg.head_dim}, vocab {cfg.vocab}, g{cfg.group})")
    return args.model if nl == cfg.num_layers else f"{args.model} ({nl} of {cfg.num_layers} layers)"


def run_reference(args):
    ws, rank, _ = dist_setup()
    if rank != 0:
        return
    cfg, model = bench_model(args)
    ctxs = lane_contexts(args, args.lanes, 0)
    # warmup steps (untimed), then K timed steps; a step is one lane-token.
    time_cpu_oracle(model, ctxs, args, 0, max_tokens=max(1, args.warmup))
    r = time_cpu_oracle(model, ctxs, args, 0, max_tokens=max(1, args.steps))
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / r["value"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": data_label(args),
        "config": {"workload": f"decode, {args.lanes} lanes, ctx U[{args.ctx_min},{args.ctx_max}], greedy "
                               "(config 5); reference step = one lane-token on the host cores",
                   "model": model_label(args, cfg, model.cfg["num_layers"]), "lanes": args.lanes},
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# this implementation
# ---------------------------------------------------------------------------

def run_glacier(args):
    import torch
    from glacier_b200 import _lib
    from glacier_b200.model import DecodeSession, DeviceModel, TensorParallelShard, tp_unique_id

    ws, rank, local = dist_setup()
    torch.cuda.set_device(local)
    pinned = pin_cores(local, ws)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    tp = args.tp
    if tp > 1 and tp != ws:
        raise SystemExit(f"--tp {tp} needs {tp} ranks (got {ws})")
    lanes = args.lanes
    # Tensor parallel: every rank serves the same lanes; lane partition: each rank its own.
    ctxs = lane_contexts(args, lanes, 0 if tp > 1 else rank)
    total_steps = args.warmup + 2 * args.steps + args.profile_steps + 4
    # The strong-scaling pass under torchrun reuses this upload for its share of rank 0's lanes.
    longest = max(int(ctxs.max()), int(lane_contexts(args, 64, 0).max()) if ws > 1 else 0)
    max_pages = -(-(longest + total_steps + 1) // 16)

    t0 = time.time()
    cfg, model = bench_model(args)
    if tp > 1:
        shard = TensorParallelShard(model, rank, tp)
        dm = DeviceModel(shard, max_positions=max_pages * 16)
        uid = [tp_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        dm.enable_tensor_parallel(rank, tp, uid[0], shard.lane_groups, shard.lane_index)
    else:
        dm = DeviceModel(model, max_positions=max_pages * 16)
    sess = DecodeSession(dm, lanes, max_pages)
    # KV: every lane's pages filled with random FP32 rows (equivalent to having
    # prefilled its context; decode cost depends only on the context length).
    g = torch.Generator(device="cuda")
    g.manual_seed(args.seed + rank)
    pages = sess.pages()
    for i in range(0, pages.shape[0], 256):
        pages[i:i + 256].normal_(generator=g)
    setup_s = time.time() - t0

    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    tokens = torch.randint(0, cfg.vocab, (lanes,), dtype=torch.int32, device=dev)
    positions = torch.from_numpy(ctxs).to(dev)
    sess.tokens.copy_(tokens)
    sess.positions.copy_(positions)

    def device_step():
        out = sess.step()
        sess.tokens.copy_(out)
        sess.positions.add_(1)

    clk = ClockSampler(local).__enter__()
    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    launches0 = _lib.lib().glacier_cuda_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.start_window()
    torch.cuda.nvtx.range_push("timed_steps")  # lets a profiler select the timed launches
    e0.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        device_step()
    enqueue_ms = (time.perf_counter() - h0) * 1e3  # host time to launch the steps (no sync inside)
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    clk.end_window()
    clk.__exit__(None, None, None)
    launches = _lib.lib().glacier_cuda_launch_count() - launches0
    dev_ms = e0.elapsed_time(e1)
    status = sess.status.cpu().numpy()
    assert (status == 0).all(), f"decode status {status}"
    assert _lib.lib().glacier_cuda_device_status(0) == 0

    # e2e: host-side runtime loop through the C ABI with pinned host buffers;
    # each step copies its inputs in and the new token ids out.
    h_tok = torch.empty(lanes, dtype=torch.int32, pin_memory=True)
    h_pos = torch.empty(lanes, dtype=torch.int32, pin_memory=True)
    h_out = torch.empty(lanes, dtype=torch.int32, pin_memory=True)
    h_tok.copy_(sess.tokens.cpu())
    h_pos.copy_(sess.positions.cpu())
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t_e2e0 = time.perf_counter()
    for _ in range(args.steps):
        sess.tokens.copy_(h_tok, non_blocking=True)
        sess.positions.copy_(h_pos, non_blocking=True)
        out = sess.step()
        h_out.copy_(out, non_blocking=True)
        stream.synchronize()
        h_tok.copy_(h_out)
        h_pos.add_(1)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t_e2e0

    # Per-kernel-class pass: the library records CUDA events on the step's stream
    # between its kernel classes for a few more steps of the same decode.
    dom = step_kernel_timing(torch, dm, sess, cfg, lanes, stream, args.profile_steps, device_step)
    sess.close()
    extras = {}
    # Multi-GPU extras (every rank takes the same collective steps in the same order):
    # the lane partition with a fixed 64-lane job, and tensor parallelism over the N ranks.
    if ws > 1 and tp == 1 and not args.no_extras:
        extras["strong_scaling"] = strong_scaling(torch, dm, cfg, args, ws, rank)
        extras["tp"] = tp_pass(torch, model, cfg, args, ws, rank)
    # Single-GPU extras (the line at N = 1): batch 1 and prefill on this upload, then the
    # other BASELINE configurations on their own synthetic models.
    if ws == 1 and not args.no_extras:
        extras["batch1"] = batch1_decode(torch, model, cfg, args, rank, stream, dm)
        extras["batch1"]["gemv_activation_modes"] = gemv_modes_timing(torch, cfg)
        extras["prefill"] = prefill_sweep(torch, dm, model, cfg, args)
    dm.close()
    if ws == 1 and not args.no_extras and not args.model_file:
        extras["gemv_config1"] = gemv_config1(torch, args)
        extras["config2"] = config2_decode(torch, args)
        extras["config3"] = config3_decode(torch, args)

    per_rank = [{"rank": rank, "ms_per_step": dev_ms / args.steps, "mean_ctx": float(ctxs.mean()),
                 "host_enqueue_ms_per_step": enqueue_ms / args.steps, "cores": pinned}]
    if ws > 1:
        gathered = [None] * ws
        torch.distributed.all_gather_object(gathered, per_rank[0])
        per_rank = gathered
    dev_ms, e2e_ms = max_over_ranks([dev_ms, e2e_s * 1e3], ws, dev)
    tokens_total = lanes * args.steps * (1 if tp > 1 else ws)
    value = tokens_total / (dev_ms / 1e3)
    e2e_value = tokens_total / (e2e_ms / 1e3)

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline:
            r = time_cpu_oracle(model, ctxs, args, args.cpu_seconds)
            cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        kv_bytes = int(np.sum(ctxs + args.warmup + args.steps // 2)) * cfg.num_layers * 2 * cfg.kv_dim * 4
        step_bytes = cfg.int4_bytes_per_token() + kv_bytes / 1  # weights once per step + every lane's KV
        peaks = load_peaks()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if tp > 1 else "weak", "vs_baseline": None,
            "dtype": "f32 activations / int4 g32 weights (fp16 scales) / f32 KV", "data": data_label(args),
            "config": {"workload": (f"decode, {lanes} lanes over {tp} tensor-parallel GPUs" if tp > 1 else
                                    f"decode, {lanes} lanes per GPU") +
                                   f", ctx U[{args.ctx_min},{args.ctx_max}], greedy (BASELINE config 5)",
                       "model": model_label(args, cfg, dm.cfg["num_layers"]),
                       "lanes_per_gpu": lanes if tp == 1 else lanes / tp,
                       "mean_ctx": float(np.mean(ctxs)),
                       "parallelism": (f"tensor parallel x{tp} (Megatron split, NCCL all-reduce of o and down)"
                                       if tp > 1 else f"lane partition x{ws} (weights replicated, no collective)"),
                       "l2": "working set (weights 4.0 GB + KV) >> 126 MB L2; no flush needed",
                       "setup_seconds": round(setup_s, 1)},
            "achieved_step_gbs": step_bytes / (dev_ms / args.steps / 1e3) / 1e9,
            "roofline": dom["roofline"],
            "kernels": dom["kernels"],
            **extras,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 2 * lanes * 4,
                    "d2h_bytes_per_step": lanes * 4},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "peaks_source": peaks.get("_source"),
            "per_rank": per_rank,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        d["_source"] = "measured (MEASURED_PEAKS.json)"
        return d
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "_source": "fallback"}


# DRAM bytes (dram__bytes_read + write) per algorithmic byte, from one ncu capture of a smaller
# case of the same kernel (profiles/); traffic scales with the K/V rows a launch reads.
DRAM_TRAFFIC_RATIO = {
    "attention": (269.894e6 / 265.1e6, "ncu dram__bytes_read.sum + dram__bytes_write.sum of the stream-K kernel "
                                       "(12 warps x 2 stages): 265.7 MB read + 4.2 MB written for 265.1 MB "
                                       "algorithmic (1 layer, 32 lanes, mean ctx 2015), scaled to this launch's K/V "
                                       "bytes"),
}

STEP_KINDS = ("embed", "norm", "proj_qkv", "rope_append", "attention", "attn_combine", "proj_o", "proj_gate_up",
              "silu", "proj_down", "lm_head", "argmax")  # glacier_cuda_step_kind order


def step_kernel_timing(torch, dm, sess, cfg, lanes, stream, steps, device_step) -> dict:
    """Per-kernel-class device time of `steps` decode steps, from CUDA events that the library
    records on the step's stream between its kernel classes, plus the roofline of the
    dominant class.  Algorithmic bytes per launch: INT4 codes (0.5 B) + fp16 scales (2 B per
    32 weights) + fp32 activations in and out for a projection; every lane's K and V rows
    (2 * kv_dim * 4 B per context position) + its query for attention; the logits for argmax."""
    import ctypes as C
    from glacier_b200 import _lib
    L = _lib.lib()
    peaks = load_peaks()
    hbm = float(peaks["hbm_gbs"])
    n = len(STEP_KINDS)
    ctx_sum = 0
    _lib.call("glacier_cuda_model_profile", dm.h, 1)
    for _ in range(steps):
        ctx_sum += int(sess.positions.sum().item()) + lanes  # context of this step = position + 1
        device_step()
    _lib.call("glacier_cuda_model_profile", dm.h, 0)
    ms = (C.c_double * n)()
    regions = (C.c_uint64 * n)()
    _lib.call("glacier_cuda_model_profile_read", dm.h, ms, regions, n)
    assert L.glacier_cuda_device_status(0) == 0
    D, F, V = cfg.dim, cfg.hidden, cfg.vocab
    nl = dm.cfg["num_layers"]

    def proj(M, K):
        return M * K // 2 + M * (K // 32) * 2 + lanes * K * 4 + lanes * M * 4

    per_launch = {
        "proj_qkv": proj(cfg.q_dim + 2 * cfg.kv_dim, D), "proj_o": proj(D, cfg.q_dim),
        "proj_gate_up": proj(2 * F, D), "proj_down": proj(D, F), "lm_head": proj(V, D),
        "attention": (ctx_sum / steps) * 2 * cfg.kv_dim * 4 + lanes * cfg.q_dim * 4,
        "argmax": lanes * V * 4,
    }
    total_ms = sum(ms[k] for k in range(n))
    kernels = {}
    for k, name in enumerate(STEP_KINDS):
        if regions[k] == 0:
            continue
        us = ms[k] / regions[k] * 1e3
        e = {"us_per_launch": us, "launches_per_step": regions[k] / steps, "share": ms[k] / total_ms}
        if name in per_launch:
            e["algorithmic_bytes"] = int(per_launch[name])
            e["gbs"] = per_launch[name] / (us * 1e-6) / 1e9
        kernels[name] = e
    dom_name = max((k for k in kernels if "gbs" in kernels[k]), key=lambda k: kernels[k]["share"])
    d = kernels[dom_name]
    what = {"attention": f"paged decode attention (attn_tma_kernel), one layer, {lanes} lanes, mean ctx "
                         f"{ctx_sum / steps / lanes:.0f}, {nl} launches per step"}.get(
        dom_name, f"{dom_name} ({nl} launches per step)")
    traffic, tsrc = None, None
    if dom_name in DRAM_TRAFFIC_RATIO:
        ratio, tsrc = DRAM_TRAFFIC_RATIO[dom_name]
        traffic = int(d["algorithmic_bytes"] * ratio)
    roof = {"bound": "hbm", "kernel": what, "achieved": d["gbs"], "peak": hbm, "unit": "GB/s",
            "frac": d["gbs"] / hbm, "traffic": traffic, "traffic_source": tsrc,
            "algorithmic_bytes": d["algorithmic_bytes"],
            "us_per_launch": d["us_per_launch"], "share_of_step": d["share"],
            "timing": "CUDA events on the decode stream around each launch, inside the library's decode step",
            "peak_source": peaks.get("_source")}
    return {"kernels": kernels, "roofline": roof}


def batch1_decode(torch, model, cfg, args, rank, stream, dm=None) -> dict:
    """Batch-1 half of the metric: one lane of the same 7B model decoding alone, on a DeviceModel
    reserved for one lane (GEMV path: 4 lanes or fewer never take the batched GEMM).  Context
    drawn like config 5's lanes; KV rows random.  Timed on the device with CUDA events over
    `steps` greedy steps; then one profiled pass gives the per-class kernel times at batch 1.
    Algorithmic bytes per token: all INT4 weights with their fp16 scales (LM head included)
    + the lane's K and V rows."""
    from glacier_b200.model import DecodeSession, DeviceModel
    ctx = int(lane_contexts(args, 1, rank)[0])
    steps, warm = 20, 3
    max_pages = -(-(ctx + steps + 2 * warm + args.profile_steps + 4) // 16)
    own = dm is None or dm.max_positions < max_pages * 16
    if own:
        dm = DeviceModel(model, max_positions=max_pages * 16)
    sess = DecodeSession(dm, 1, max_pages)  # one reserved lane: the GEMV path
    g = torch.Generator(device="cuda")
    g.manual_seed(args.seed + 1000 + rank)
    pages = sess.pages()
    for i in range(0, pages.shape[0], 256):
        pages[i:i + 256].normal_(generator=g)
    sess.tokens.fill_(1)
    sess.positions.fill_(ctx)

    def step():
        out = sess.step()
        sess.tokens.copy_(out)
        sess.positions.add_(1)

    # The timed steps replay the greedy step as a CUDA graph on a side stream.
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for _ in range(warm):
            step()
        sess.capture_greedy_step(stream=side)
        for _ in range(warm):
            sess.replay_greedy_step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(side)
        for _ in range(steps):
            sess.replay_greedy_step()
        e1.record(side)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    assert (sess.status.cpu().numpy() == 0).all()
    kv = (ctx + warm + steps // 2) * cfg.num_layers * 2 * cfg.kv_dim * 4
    byt = cfg.int4_bytes_per_token() + kv
    hbm = float(load_peaks()["hbm_gbs"])
    prof = step_kernel_timing(torch, dm, sess, cfg, 1, stream, args.profile_steps, step)
    sess.close()
    if own:
        dm.close()
    cpu = time_cpu_oracle(model, np.array([ctx], np.int32), args, min(args.cpu_seconds, 4.0))
    return {"tok_s": 1e3 / ms, "ms_per_token": ms, "ctx": ctx, "algorithmic_bytes_per_token": int(byt),
            "achieved_gbs": byt / (ms * 1e-3) / 1e9, "frac_of_hbm_peak": byt / (ms * 1e-3) / 1e9 / hbm,
            "roofline": {"bound": "hbm", "achieved": byt / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": byt / (ms * 1e-3) / 1e9 / hbm, "algorithmic_bytes": int(byt)},
            "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "timing": f"CUDA events over {steps} CUDA-graph replays of the greedy step after {warm} warm-up steps",
            "kernels": prof["kernels"]}


def gemv_modes_timing(torch, cfg) -> dict:
    """The batch-1 INT4 GEMV on the 7B projection shapes in both activation modes: FP32
    activations (glacier_cuda_int4_linear, the parity mode of the decode step) and Q8
    activations (glacier_cuda_int4_linear_q8, the reference's default decode numerics,
    bit-identical to its portable path).  Each figure is one replay of a CUDA graph of 20
    back-to-back calls on rotating weight copies (more than L2 in total), timed with CUDA events
    on the capture stream; bytes are the INT4 codes plus fp16 scales."""
    from glacier_b200 import _lib
    L = _lib.lib()
    out = {}
    shapes = {"qkv": (cfg.q_dim + 2 * cfg.kv_dim, cfg.dim), "o": (cfg.dim, cfg.q_dim), "gate_up": (2 * cfg.hidden, cfg.dim)}
    st = torch.cuda.Stream()
    for name, (M, K) in shapes.items():
        n = M * K
        copies = max(2, min(8, int(4 * 126e6 // (n * 0.5625)) + 1))
        Ws = [torch.randint(0, 256, (n // 2,), dtype=torch.uint8, device="cuda") for _ in range(copies)]
        Ss = [(torch.rand(n // 32, device="cuda") * 0.02).half() for _ in range(copies)]
        x = torch.randn(1, K, device="cuda")
        y = torch.empty(1, M, device="cuda")
        byt = n // 2 + n // 32 * 2
        e = {}
        for mode, fn in (("fp32", L.glacier_cuda_int4_linear), ("q8", L.glacier_cuda_int4_linear_q8)):
            def call(i):
                assert fn(x.data_ptr(), 1, Ws[i % copies].data_ptr(), Ss[i % copies].data_ptr(), 1, None, y.data_ptr(),
                          M, K, 32, st.cuda_stream) == 0
            with torch.cuda.stream(st):
                for i in range(3):
                    call(i)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st):
                    for i in range(20):
                        call(i)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                g.replay()
                e1.record(st)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / 20 * 1e3
            e[mode] = {"us": us, "gbs": byt / (us * 1e-6) / 1e9}
            del g
        out[f"{name}_{M}x{K}"] = e
    return out


def _graph_time_us(torch, stream, call, n: int) -> float:
    """Mean device time of `call(i)` over one replay of a CUDA graph of n back-to-back calls
    (after a warm replay), CUDA events on the capture stream."""
    with torch.cuda.stream(stream):
        for i in range(3):
            call(i)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                call(i)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / n * 1e3


def gemv_config1(torch, args) -> dict:
    """Config 1, the reference's kernel microbench shape (bench/int4_kernel.zig:18-30): one
    4864 x 896 INT4 g32 GEMV, y = x * dequant(W)^T, x ~ N(0, 1) fp32, uniform codes, fp16 scales
    of |N(0, 0.02)|.  The matrix is 2.47 MB, inside the 126 MB L2, so the timed loop walks
    rotating copies uploaded once through the persistent weight handle (fp16 scale rows padded
    for TMA), more than 4x L2 in total, as one CUDA graph of 600 calls.  Algorithmic bytes per
    call: codes + fp16 scales + x + y = 2,474,496.  CPU baseline: the oracle's
    linearInt4OnTheFly on 1 thread and with the reference's row split over all host threads."""
    import ctypes as C
    import oracle
    from glacier_b200 import _lib
    from glacier_b200.model import random_int4
    L = _lib.lib()
    M, K, G = 4864, 896, 32
    rng = np.random.default_rng(args.seed + 11)
    packed, s32 = random_int4(rng, M, K, G)
    s16 = s32.astype(np.float16).view(np.uint16)
    x = rng.standard_normal(K, dtype=np.float32)
    wbytes = M * K // 2 + M * K // G * 2
    byt = wbytes + 4 * K + 4 * M
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    copies = int(4 * l2 // wbytes) + 1
    ctx = _lib.handle(L.glacier_cuda_context_create(torch.cuda.current_device()))
    hs = []
    try:
        for _ in range(copies):
            hs.append(_lib.handle(L.glacier_cuda_int4_weight_create_ex(
                ctx, packed.ctypes.data, packed.size, s16.ctypes.data, s16.size, 1, G, K, M)))
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty(M, dtype=torch.float32, device="cuda")
        st = torch.cuda.Stream()

        def call(i):
            assert L.glacier_cuda_int4_weight_matvec(hs[i % copies], xd.data_ptr(), yd.data_ptr(), None,
                                                     C.c_void_p(st.cuda_stream)) == 0

        us = _graph_time_us(torch, st, call, 600)
        y = yd.cpu().numpy()
    finally:
        for h in hs:
            L.glacier_cuda_int4_weight_destroy(h)
        L.glacier_cuda_context_destroy(ctx)
    ref = oracle.linear_int4(x, packed, s32, M, K, G)[0]
    err = float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))
    hbm = float(load_peaks()["hbm_gbs"])
    cpu = {}
    for th in (1, cpu_threads()):
        reps, t = 0, 0.0
        while t < 1.0:
            t0 = time.perf_counter()
            oracle.linear_int4(x, packed, s32, M, K, G, threads=th)
            t += time.perf_counter() - t0
            reps += 1
        cpu[th] = t / reps * 1e6
    return {
        "us": us, "gbs": byt / (us * 1e-6) / 1e9,
        "config": f"4864x896 INT4 g32, fp16 scales, batch 1; {copies} rotating copies "
                  f"({copies * wbytes / 1e6:.0f} MB > 4x L2), CUDA graph of 600 calls",
        "max_err_vs_row_max": err,
        "roofline": {"bound": "hbm", "achieved": byt / (us * 1e-6) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": byt / (us * 1e-6) / 1e9 / hbm, "algorithmic_bytes": byt},
        "cpu_baseline": {"value": cpu[1], "unit": "us per GEMV", "cores": 1, "kind": "port",
                         "all_cores_us": cpu[cpu_threads()], "all_cores": cpu_threads(),
                         "sample": "the oracle's linearInt4OnTheFly on the same matrix and input, repeated for "
                                   "about 1 s per thread count (row split over all host threads for all_cores)"},
    }


def _random_pages(torch, sess, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    pages = sess.pages()
    for i in range(0, pages.shape[0], 256):
        pages[i:i + 256].normal_(generator=g)


def _graph_decode(torch, sess, warm: int, steps: int) -> float:
    """ms per greedy step: `warm` stream steps, then a CUDA graph of one greedy step replayed
    `warm` times untimed and `steps` times timed (CUDA events on the side stream)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warm):
            out = sess.step(stream=side)
            sess.tokens.copy_(out)
            sess.positions.add_(1)
        sess.capture_greedy_step(stream=side)
        for _ in range(warm):
            sess.replay_greedy_step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(side)
        for _ in range(steps):
            sess.replay_greedy_step()
        e1.record(side)
    torch.cuda.synchronize()
    assert (sess.status.cpu().numpy() == 0).all()
    return e0.elapsed_time(e1) / steps


def config2_decode(torch, args) -> dict:
    """Config 2: the 0.5B model (24 layers, D 896, FFN 4864, 14/2 heads of 64, vocab 151936),
    batch 1: a 512-token prompt of uniform ids through glacier_cuda_prefill, then 128 greedy
    tokens (CUDA-graph replays of the greedy step after 3 warm-up tokens).  Algorithmic bytes
    per token: every INT4 code and fp16 scale (LM head included) + the lane's K/V rows."""
    from glacier_b200.model import PRESETS, DecodeSession, DeviceModel, SyntheticModel
    cfg = PRESETS["qwen2.5-0.5b"]
    m = SyntheticModel(cfg, seed=args.seed + 2)
    prompt_len, new, warm = 512, 128, 3
    max_pages = -(-(prompt_len + new + 2 * warm + 2) // 16)
    dm = DeviceModel(m, max_positions=max_pages * 16)
    sess = DecodeSession(dm, 1, max_pages)
    rng = np.random.default_rng(args.seed + 3)
    prompt = rng.integers(0, cfg.vocab, size=prompt_len).astype(np.int32)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    tok = sess.prefill(prompt)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    assert int(sess.last_status.cpu()[0]) == 0
    sess.tokens.copy_(tok)
    sess.positions.fill_(prompt_len)
    ms = _graph_decode(torch, sess, warm, new)
    mean_ctx = prompt_len + 2 * warm + new / 2
    byt = cfg.int4_bytes_per_token() + int(mean_ctx) * cfg.num_layers * 2 * cfg.kv_dim * 4
    hbm = float(load_peaks()["hbm_gbs"])
    sess.close()
    dm.close()
    cpu = time_cpu_oracle(m, np.array([prompt_len + new // 2], np.int32), args, min(args.cpu_seconds, 4.0))
    return {
        "tok_s": 1e3 / ms, "ms_per_token": ms, "prefill_512_ms": prefill_ms,
        "config": "0.5B shape, batch 1, 512-token uniform prompt (chunked prefill on the one-lane GEMV "
                  "path), then 128 greedy tokens; CUDA-graph replays of the greedy step",
        "algorithmic_bytes_per_token": int(byt),
        "roofline": {"bound": "hbm", "achieved": byt / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": byt / (ms * 1e-3) / 1e9 / hbm},
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
    }


def config3_decode(torch, args) -> dict:
    """Config 3: the 1.5B model (28 layers, D 1536, FFN 8960, 12/2 heads of 128, vocab 151936),
    8 lanes with contexts U[128, 2048] (random FP32 K/V rows up to each lane's context), greedy,
    256 tokens per lane (CUDA-graph replays of the greedy step after 3 warm-up steps).
    Algorithmic bytes per step: the weights once + every lane's K/V rows."""
    from glacier_b200.model import PRESETS, DecodeSession, DeviceModel, SyntheticModel
    cfg = PRESETS["qwen2.5-1.5b"]
    m = SyntheticModel(cfg, seed=args.seed + 4)
    lanes, steps, warm = 8, 256, 3
    rng = np.random.default_rng(args.seed + 5)
    ctxs = rng.integers(128, 2049, size=lanes).astype(np.int32)
    max_pages = -(-(int(ctxs.max()) + steps + 2 * warm + 2) // 16)
    dm = DeviceModel(m, max_positions=max_pages * 16)
    sess = DecodeSession(dm, lanes, max_pages)
    _random_pages(torch, sess, args.seed + 6)
    sess.tokens.copy_(torch.from_numpy(rng.integers(0, cfg.vocab, size=lanes).astype(np.int32)))
    sess.positions.copy_(torch.from_numpy(ctxs))
    ms = _graph_decode(torch, sess, warm, steps)
    kv = int(np.sum(ctxs + 2 * warm + steps // 2)) * cfg.num_layers * 2 * cfg.kv_dim * 4
    byt = cfg.int4_bytes_per_token() + kv
    hbm = float(load_peaks()["hbm_gbs"])
    sess.close()
    dm.close()
    cpu = time_cpu_oracle(m, ctxs, args, min(args.cpu_seconds, 4.0))
    return {
        "tok_s": lanes * 1e3 / ms, "ms_per_step": ms, "lanes": lanes, "mean_ctx": float(np.mean(ctxs)),
        "config": "1.5B shape, 8 lanes, ctx U[128,2048], greedy 256 tokens per lane (tcgen05 GEMM path); "
                  "CUDA-graph replays of the greedy step",
        "algorithmic_bytes_per_step": int(byt),
        "roofline": {"bound": "hbm", "achieved": byt / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": byt / (ms * 1e-3) / 1e9 / hbm},
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
    }


def prefill_flops(cfg, nl: int, T: int) -> float:
    """Useful FLOPs of a T-token prompt: 2 x linear params x T + causal attention (QK and PV)."""
    lin = nl * ((cfg.q_dim + 2 * cfg.kv_dim) * cfg.dim + cfg.dim * cfg.q_dim + 3 * cfg.hidden * cfg.dim)
    return 2.0 * lin * T + nl * 4.0 * cfg.head_dim * cfg.num_heads * T * (T + 1) / 2


def prefill_sweep(torch, dm, model, cfg, args) -> dict:
    """Config 4 on the bench's own 7B upload: one prompt of T = 128, 512 and 2048 uniform ids,
    chunks of 128 rows on the tcgen05 GEMM, timed on the device (1 warm-up, 3 timed prompts).
    MFU against the measured dense bf16 peak.  CPU baseline: the reference feeds g32 prompts one
    token at a time (generate.zig:2377), so its prompt rate is its per-token rate, timed on the
    oracle at a context of 256."""
    from glacier_b200.model import DecodeSession
    peaks = load_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0)) * 1e12
    nl = dm.cfg["num_layers"]
    out = {}
    for T in (128, 512, 2048):
        sess = DecodeSession(dm, 1, -(-(T + 1) // 16), reserve_lanes=128)
        prompt = torch.from_numpy(np.random.default_rng(args.seed + T).integers(0, cfg.vocab, size=T)
                                  .astype(np.int32)).cuda()
        sess.prefill(prompt)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            sess.prefill(prompt)
        e1.record()
        torch.cuda.synchronize()
        assert int(sess.last_status.cpu()[0]) == 0
        ms = e0.elapsed_time(e1) / 3
        fl = prefill_flops(cfg, nl, T)
        out[f"T{T}"] = {"tok_s": T / (ms / 1e3), "ms": ms,
                        "roofline": {"bound": "tensor", "achieved": fl / (ms / 1e3) / 1e12, "peak": peak / 1e12,
                                     "unit": "TFLOP/s", "frac": fl / (ms / 1e3) / peak}}
        sess.close()
    cpu = time_cpu_oracle(model, np.array([256], np.int32), args, min(args.cpu_seconds, 4.0))
    out["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind")}
    out["cpu_baseline"]["sample"] = ("prompt tokens fed one at a time (the reference's g32 prompt path) at context "
                                     "256: " + cpu["sample"])
    out["note"] = ("useful FLOPs (MFU); the exact fp16 hi/lo operand split runs 3x the MMA work; "
                   "peak " + str(peaks.get("_source")))
    return out


def strong_scaling(torch, dm, cfg, args, ws, rank, lanes_total: int = 64) -> dict:
    """Lane partition with a fixed job: `lanes_total` lanes (contexts drawn like the headline's)
    split over the N ranks, each rank decoding its share on its full weight replica; whole-job
    tok/s from the max over ranks of the device time of `args.steps` steps."""
    from glacier_b200.model import DecodeSession
    per = -(-lanes_total // ws)
    lanes = max(0, min(per, lanes_total - rank * per))
    all_ctx = lane_contexts(args, lanes_total, 0)
    ctxs = all_ctx[rank * per:rank * per + lanes]
    ms = 0.0
    sess = None
    if lanes:
        max_pages = -(-(int(ctxs.max()) + args.warmup + args.steps + 2) // 16)
        sess = DecodeSession(dm, lanes, max_pages)
        _random_pages(torch, sess, args.seed + 77 + rank)
        sess.tokens.fill_(1)
        sess.positions.copy_(torch.from_numpy(ctxs))
        for _ in range(args.warmup):
            out = sess.step()
            sess.tokens.copy_(out)
            sess.positions.add_(1)
    torch.cuda.synchronize()
    torch.distributed.barrier()
    torch.cuda.synchronize()
    if sess is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            out = sess.step()
            sess.tokens.copy_(out)
            sess.positions.add_(1)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        assert (sess.status.cpu().numpy() == 0).all()
        sess.close()
    (ms,) = max_over_ranks([ms], ws, torch.device("cuda", torch.cuda.current_device()))
    return {"lanes_total": lanes_total, "lanes_per_gpu": per, "tok_s": lanes_total * args.steps / (ms / 1e3),
            "ms_per_step": ms / args.steps, "scaling": "strong",
            "timing": "device time of the timed steps, CUDA events, max over ranks"}


def tp_pass(torch, model, cfg, args, ws, rank) -> dict:
    """Tensor parallelism over the N ranks (Megatron split: each rank holds H/N q heads, Hkv/N kv
    heads, F/N FFN rows and the matching o / down columns; an NCCL all-reduce after o and after
    down; with more ranks than kv heads, N/Hkv ranks share a kv-head group and split its lanes):
    one 64-lane job with the headline's contexts.  Reports whole-job tok/s (max over
    ranks of the device time) and the all-reduce share of the profiled step."""
    import ctypes as C
    from glacier_b200 import _lib
    from glacier_b200.model import DecodeSession, DeviceModel, TensorParallelShard, tp_unique_id
    try:
        shard = TensorParallelShard(model, rank, ws)
    except ValueError as e:
        return {"unavailable": str(e)}
    lanes = 64
    ctxs = lane_contexts(args, lanes, 0)
    max_pages = -(-(int(ctxs.max()) + args.warmup + args.steps + args.profile_steps + 2) // 16)
    dm = DeviceModel(shard, max_positions=max_pages * 16)
    uid = [tp_unique_id() if rank == 0 else None]
    torch.distributed.broadcast_object_list(uid, src=0)
    dm.enable_tensor_parallel(rank, ws, uid[0], shard.lane_groups, shard.lane_index)
    sess = DecodeSession(dm, lanes, max_pages)
    _random_pages(torch, sess, args.seed + 99 + rank)
    sess.tokens.fill_(1)
    sess.positions.copy_(torch.from_numpy(ctxs))

    def step():
        out = sess.step()
        sess.tokens.copy_(out)
        sess.positions.add_(1)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # Per-class device time of a few more steps: the all-reduce share.
    n = len(STEP_KINDS) + 1
    _lib.call("glacier_cuda_model_profile", dm.h, 1)
    for _ in range(args.profile_steps):
        step()
    _lib.call("glacier_cuda_model_profile", dm.h, 0)
    cms = (C.c_double * n)()
    regions = (C.c_uint64 * n)()
    _lib.call("glacier_cuda_model_profile_read", dm.h, cms, regions, n)
    share = cms[n - 1] / max(sum(cms), 1e-30)
    assert (sess.status.cpu().numpy() == 0).all()
    sess.close()
    dm.close()
    ms, share = max_over_ranks([ms, share], ws, torch.device("cuda", torch.cuda.current_device()))
    return {"lanes": lanes, "tp": ws, "tok_s": lanes * args.steps / (ms / 1e3), "ms_per_step": ms / args.steps,
            "all_reduce_share": share, "scaling": "strong",
            "parallelism": f"tensor parallel x{ws} (Megatron split, NCCL all-reduce of o and down, 2 per layer"
                           + (f"; {shard.lane_groups} ranks per kv-head group split its lanes)" if shard.lane_groups > 1
                              else ")")}


def run_prefill(args):
    """Config 4: one prompt of T tokens through the 7B model (chunks of 128 rows on the
    tensor-core GEMM), timed on the device; reports prompt tok/s and MFU against the measured
    dense bf16 peak (useful FLOPs: 2 x 6.525e9 linear params x T + 200,704 x T^2 causal attention)."""
    import torch
    from glacier_b200 import _lib
    from glacier_b200.model import DecodeSession, DeviceModel
    ws, rank, local = dist_setup()
    torch.cuda.set_device(local)
    T = args.tokens
    max_pages = -(-(T + 1) // 16)
    cfg, model = bench_model(args)
    dm = DeviceModel(model, max_positions=max_pages * 16)
    sess = DecodeSession(dm, 1, max_pages, reserve_lanes=128)
    rng = np.random.default_rng(args.seed + rank)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab, size=T).astype(np.int32)).cuda()
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        sess.prefill(prompt)
    torch.cuda.synchronize()
    launches0 = _lib.lib().glacier_cuda_launch_count()
    clk = ClockSampler(local).__enter__()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    clk.start_window()
    e0.record(stream)
    for _ in range(args.steps):
        sess.prefill(prompt)
    e1.record(stream)
    torch.cuda.synchronize()
    clk.end_window()
    clk.__exit__(None, None, None)
    launches = _lib.lib().glacier_cuda_launch_count() - launches0
    assert int(sess.last_status.cpu()[0]) == 0 and _lib.lib().glacier_cuda_device_status(0) == 0
    ms = e0.elapsed_time(e1) / args.steps
    # e2e: prompt ids copied from pinned host memory, the next token read back, every prefill.
    h_prompt = prompt.cpu().pin_memory()
    h_out = torch.empty(1, dtype=torch.int32, pin_memory=True)
    d_prompt = torch.empty_like(prompt)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        d_prompt.copy_(h_prompt, non_blocking=True)
        h_out.copy_(sess.prefill(d_prompt), non_blocking=True)
        stream.synchronize()
    e2e_s = (time.perf_counter() - t0) / args.steps
    nl = dm.cfg["num_layers"]
    lin_params = nl * ((cfg.q_dim + 2 * cfg.kv_dim) * cfg.dim + cfg.dim * cfg.q_dim + 3 * cfg.hidden * cfg.dim)
    flops = 2.0 * lin_params * T + nl * 4.0 * cfg.head_dim * cfg.num_heads * T * (T + 1) / 2
    peaks = load_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0)) * 1e12
    line = {
        "metric": "INT4 prompt prefill tok/s (Qwen2.5-7B shape, one request)", "value": T / (ms / 1e3),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 activations / int4 g32 weights (fp16 scales) / f32 KV; fp16 hi/lo tensor-core operands",
        "data": data_label(args), "config": {"workload": f"7B prefill, T={T} (BASELINE config 4)", "model": args.model,
                                        "tokens": T, "layers": nl, "chunk_rows": 128},
        "roofline": {"bound": "tensor", "achieved": flops / (ms / 1e3) / 1e12, "peak": peak / 1e12,
                     "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / peak, "traffic": None,
                     "note": "useful FLOPs (MFU); the exact fp16 hi/lo operand split runs 3x the MMA work",
                     "peak_source": peaks.get("_source")},
        "e2e": {"value": T / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * T, "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches), "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    sess.close()
    dm.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    else:
        run_glacier(args)


if __name__ == "__main__":
    main()
