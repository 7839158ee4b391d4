"""Full decode step (all kernels + the C++ runtime) vs the CPU oracle.

Greedy token ids must match the oracle exactly except at near-ties: a step whose
oracle top-2 logit gap is below 1e-3 * max(1, |top1|) is exempt, and the lane
stops being compared after such a step (its continuation legitimately differs).
Logits must match within DECODE_LOGIT_TOL of the row's largest |logit| (the
kernels' own per-element 1e-3 bound is checked by their tests; through several
layers their rounding compounds onto logits near zero).
"""
import numpy as np
import pytest

import oracle
from helpers import DECODE_LOGIT_TOL, max_err_vs_row_max

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def near_tie(logits) -> bool:
    top2 = np.sort(logits)[-2:]
    return (top2[1] - top2[0]) < 1e-3 * max(1.0, abs(float(top2[1])))


def run_parity(cfg, lanes, prompt_len, new_tokens, seed=7):
    from glacier_b200.model import DecodeSession, DeviceModel, SyntheticModel
    m = SyntheticModel(cfg, seed=seed)
    max_pages = -(-(prompt_len + new_tokens) // 16)
    dm = DeviceModel(m, max_positions=max_pages * 16)
    sess = DecodeSession(dm, lanes, max_pages)
    om = oracle.OracleModel(m, rope_positions=max_pages * 16, threads=4)
    pf = om.page_floats()
    pools = [np.zeros(max_pages * pf, np.float32) for _ in range(lanes)]
    bt = np.arange(max_pages, dtype=np.int32)
    rng = np.random.default_rng(seed)
    prompts = rng.integers(0, cfg.vocab, size=(lanes, prompt_len)).astype(np.int32)
    logits_dev = torch.empty((lanes, cfg.vocab), dtype=torch.float32, device="cuda")
    live = [True] * lanes
    compared = 0
    cur = prompts[:, 0].copy()
    for pos in range(prompt_len + new_tokens - 1):
        out = sess.step(tokens=cur, positions=[pos] * lanes, logits=logits_dev)
        gpu_tok = out.cpu().numpy()
        assert sess.status.cpu().numpy().tolist() == [0] * lanes
        gl = logits_dev.cpu().numpy()
        for b in range(lanes):
            ol, _ = om.decode_token(pools[b], bt, pos, int(cur[b]))
            if not live[b]:
                continue
            assert max_err_vs_row_max(gl[b], ol) <= DECODE_LOGIT_TOL, (b, pos)
            if pos >= prompt_len - 1:
                ref_tok = oracle.argmax(ol)
                if gpu_tok[b] != ref_tok:
                    assert near_tie(ol), (b, pos, gpu_tok[b], ref_tok)
                    live[b] = False
                else:
                    compared += 1
        # Prompt tokens first (token-at-a-time prefill, the reference's g32 path),
        # then each lane's own greedy output.
        cur = prompts[:, pos + 1].copy() if pos + 1 < prompt_len else gpu_tok.astype(np.int32)
    sess.close()
    dm.close()
    return compared


def test_decode_small_gqa_model():
    from glacier_b200.model import ModelConfig
    cfg = ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)
    assert run_parity(cfg, lanes=3, prompt_len=20, new_tokens=6) >= 12


def test_decode_7b_head_geometry():
    from glacier_b200.model import ModelConfig
    cfg = ModelConfig(num_layers=2, dim=512, hidden=1024, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048)
    assert run_parity(cfg, lanes=2, prompt_len=18, new_tokens=4) >= 6


@pytest.mark.parametrize("lanes", [1, 2])
def test_decode_7b_layer_shapes_gemv_mode(lanes):
    """One layer at the full 7B shapes in GEMV mode (cluster K-split GEMVs, the SwiGLU folded
    into the 3584 x 18944 down projection)."""
    from glacier_b200.model import ModelConfig
    cfg = ModelConfig(num_layers=1, dim=3584, hidden=18944, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048)
    assert run_parity(cfg, lanes=lanes, prompt_len=3, new_tokens=3) >= 3 * lanes


def test_decode_05b_head_geometry_batch5():
    from glacier_b200.model import ModelConfig
    # five lanes: the tensor-core GEMV runs as a 4-row launch plus a 1-row launch
    cfg = ModelConfig(num_layers=1, dim=896, hidden=1024, num_heads=14, num_kv_heads=2, head_dim=64, vocab=1536)
    assert run_parity(cfg, lanes=5, prompt_len=3, new_tokens=3) >= 10


def test_decode_tensor_core_mode_16_lanes():
    from glacier_b200.model import ModelConfig
    # more than 4 lanes: every projection runs the tcgen05 GEMM with split-K partials
    cfg = ModelConfig(num_layers=2, dim=512, hidden=1024, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048)
    assert run_parity(cfg, lanes=16, prompt_len=4, new_tokens=3) >= 30


@pytest.mark.parametrize("lanes", [1, 8])
def test_greedy_step_graph_replay_matches_stream_steps(lanes):
    """A CUDA-graph replay of the greedy step produces the same token ids, step for step, as
    launching the step on the stream (GEMV path for 1 lane, tensor-core GEMM for 8)."""
    from glacier_b200.model import DecodeSession, DeviceModel, ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=2, dim=512, hidden=1024, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048)
    dm = DeviceModel(SyntheticModel(cfg, seed=5), max_positions=128)
    sess = DecodeSession(dm, lanes, 8)
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    sess.pages().normal_(generator=g)
    start_tok = torch.arange(3, 3 + lanes, dtype=torch.int32, device="cuda")
    start_pos = torch.full((lanes,), 40, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        sess.tokens.copy_(start_tok)
        sess.positions.copy_(start_pos)
        plain = []
        for _ in range(5):
            out = sess.step(stream=s)
            sess.tokens.copy_(out)
            sess.positions.add_(1)
            plain.append(out.cpu().tolist())
        sess.capture_greedy_step(stream=s)
        sess.tokens.copy_(start_tok)
        sess.positions.copy_(start_pos)
        replayed = []
        for _ in range(5):
            replayed.append(sess.replay_greedy_step().cpu().tolist())
    torch.cuda.synchronize()
    assert replayed == plain
    assert sess.status.cpu().tolist() == [0] * lanes
    sess.close()
    dm.close()


def test_decode_tensor_core_mode_group16_model():
    from glacier_b200.model import ModelConfig
    # the reference's production g16 layout on the tcgen05 GEMM (16 lanes)
    cfg = ModelConfig(num_layers=2, dim=512, hidden=1024, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048,
                      group=16)
    assert run_parity(cfg, lanes=16, prompt_len=4, new_tokens=3) >= 30


def test_step_profile_counts_every_kernel_class():
    """The per-class event timing sees each class the expected number of times per step and
    leaves the step's results unchanged."""
    import ctypes as C
    from glacier_b200 import _lib
    from glacier_b200.model import DecodeSession, DeviceModel, ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=2, dim=512, hidden=1024, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048)
    dm = DeviceModel(SyntheticModel(cfg, seed=3), max_positions=64)
    sess = DecodeSession(dm, 8, 4)
    toks = [5, 6, 7, 8, 9, 10, 11, 12]
    plain = sess.step(tokens=toks, positions=[3] * 8).cpu().tolist()
    _lib.call("glacier_cuda_model_profile", dm.h, 1)
    steps = 3
    for _ in range(steps):
        got = sess.step(tokens=toks, positions=[3] * 8).cpu().tolist()
        assert got == plain
    _lib.call("glacier_cuda_model_profile", dm.h, 0)
    n = 12
    ms, regions = (C.c_double * n)(), (C.c_uint64 * n)()
    _lib.call("glacier_cuda_model_profile_read", dm.h, ms, regions, n)
    per_step = [r // steps for r in regions]
    L = cfg.num_layers
    # embed, norm (2 per layer + final), qkv, rope, attention, combine, o, gate_up, silu, down, lm_head, argmax
    assert per_step == [1, 2 * L + 1, L, L, L, L, L, L, L, L, 1, 1]
    assert all(ms[k] > 0 for k in range(n))
    # A second read without new steps reports nothing.
    _lib.call("glacier_cuda_model_profile_read", dm.h, ms, regions, n)
    assert list(regions) == [0] * n
    sess.close()
    dm.close()


def _prefill_parity(cfg, reserve_lanes, prompt_len, new_tokens, seed=11):
    """Chunked prefill of one prompt, then greedy decode steps, against the oracle's
    token-at-a-time prompt loop (the reference's path for g32)."""
    from glacier_b200.model import DecodeSession, DeviceModel, SyntheticModel
    m = SyntheticModel(cfg, seed=seed)
    max_pages = -(-(prompt_len + new_tokens) // 16)
    dm = DeviceModel(m, max_positions=max_pages * 16)
    sess = DecodeSession(dm, 1, max_pages, reserve_lanes=reserve_lanes)
    om = oracle.OracleModel(m, rope_positions=max_pages * 16, threads=4)
    pool = np.zeros(max_pages * om.page_floats(), np.float32)
    bt = np.arange(max_pages, dtype=np.int32)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg.vocab, size=prompt_len).astype(np.int32)
    for pos in range(prompt_len):
        ol, _ = om.decode_token(pool, bt, pos, int(prompt[pos]))
    logits_dev = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    tok = int(sess.prefill(prompt, logits=logits_dev).cpu()[0])
    assert int(sess.last_status.cpu()[0]) == 0
    assert max_err_vs_row_max(logits_dev.cpu().numpy(), ol) <= DECODE_LOGIT_TOL
    ref = oracle.argmax(ol)
    if tok != ref:
        assert near_tie(ol)
        return 0
    compared = 1
    cur, pos = tok, prompt_len
    step_logits = torch.empty((1, cfg.vocab), dtype=torch.float32, device="cuda")
    for _ in range(new_tokens - 1):
        out = int(sess.step(tokens=[cur], positions=[pos], logits=step_logits).cpu()[0])
        ol, _ = om.decode_token(pool, bt, pos, cur)
        assert max_err_vs_row_max(step_logits.cpu().numpy()[0], ol) <= DECODE_LOGIT_TOL, pos
        ref = oracle.argmax(ol)
        if out != ref:
            assert near_tie(ol)
            break
        compared += 1
        cur, pos = out, pos + 1
    sess.close()
    dm.close()
    return compared


def test_prefill_chunks_on_tensor_cores_then_decode():
    from glacier_b200.model import ModelConfig
    # 16 reserved lanes: tensor-core projections; 40 prompt tokens = chunks of 16, 16 and 8
    cfg = ModelConfig(num_layers=2, dim=512, hidden=1024, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048)
    assert _prefill_parity(cfg, reserve_lanes=16, prompt_len=40, new_tokens=4) >= 2


def test_prefill_chunks_on_gemv_path():
    from glacier_b200.model import ModelConfig
    # 4 reserved lanes: GEMV projections; 19 prompt tokens = chunks of 4 (x4) and 3
    cfg = ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)
    assert _prefill_parity(cfg, reserve_lanes=4, prompt_len=19, new_tokens=3) >= 2


def test_model_load_qio_equals_direct_upload():
    """glacier_cuda_model_load_qio takes the reference's qio page payload (qio.zig:73 encodePage:
    16-byte sub-header, f32 scales, packed nibbles) as the oracle's gor_qio_encode writes it.  A
    model loaded from payloads decodes bit-identically to the same model loaded from the
    quantizer's (packed, scales), both match the oracle, and malformed payloads are rejected
    before any write."""
    import ctypes as C
    from glacier_b200 import _lib
    from glacier_b200.model import DecodeSession, DeviceModel, ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)
    m = SyntheticModel(cfg, seed=17)
    rng = np.random.default_rng(17)
    payloads = {}
    shapes = {"wq": (cfg.q_dim, cfg.dim), "wk": (cfg.kv_dim, cfg.dim), "wv": (cfg.kv_dim, cfg.dim),
              "wo": (cfg.dim, cfg.q_dim), "wg": (cfg.hidden, cfg.dim), "wu": (cfg.hidden, cfg.dim),
              "wd": (cfg.dim, cfg.hidden)}
    kinds = {"wq": _lib.W_Q, "wk": _lib.W_K, "wv": _lib.W_V, "wo": _lib.W_O, "wg": _lib.W_GATE, "wu": _lib.W_UP,
             "wd": _lib.W_DOWN}
    for i, L in enumerate(m.layers):
        for key, (o, k) in shapes.items():
            w = rng.standard_normal(o * k, dtype=np.float32) * np.float32(0.05)
            L[key] = oracle.quantize(w, 32)
            payloads[(i, kinds[key])] = oracle.qio_encode(w, 32)
    w = rng.standard_normal(cfg.vocab * cfg.dim, dtype=np.float32) * np.float32(0.05)
    m.lm_head = oracle.quantize(w, 32)
    payloads[(-1, _lib.W_LM_HEAD)] = oracle.qio_encode(w, 32)
    # The payload is header + the quantizer's scales + its packed codes, byte for byte.
    for (i, kind), pl in payloads.items():
        packed, scales = m.lm_head if i < 0 else m.layers[i][[k for k, v in kinds.items() if v == kind][0]]
        assert pl[16:16 + 4 * scales.size] == scales.tobytes() and pl[16 + 4 * scales.size:] == packed.tobytes()

    class QioDeviceModel(DeviceModel):
        def _int4(self, layer, kind, packed, scales):
            pl = np.frombuffer(payloads[(layer, kind)], np.uint8)
            _lib.call("glacier_cuda_model_load_qio", self.h, layer, kind, pl.ctypes.data, pl.size)

    # The quantizer's scales are arbitrary f32 values: both models keep them in f32 (no fp16
    # mirror), as the oracle computes.
    da, db = DeviceModel(m, 64, scales_f16=False), QioDeviceModel(m, 64, scales_f16=False)
    sa, sb = DecodeSession(da, 2, 4), DecodeSession(db, 2, 4)
    om = oracle.OracleModel(m, rope_positions=64, threads=4)
    pools = [np.zeros(4 * om.page_floats(), np.float32) for _ in range(2)]
    bt = np.arange(4, dtype=np.int32)
    la = torch.empty((2, cfg.vocab), dtype=torch.float32, device="cuda")
    lb = torch.empty_like(la)
    cur = np.array([3, 900], np.int32)
    for pos in range(5):
        ta = sa.step(tokens=cur, positions=[pos] * 2, logits=la).cpu().numpy()
        tb = sb.step(tokens=cur, positions=[pos] * 2, logits=lb).cpu().numpy()
        assert la.cpu().numpy().tobytes() == lb.cpu().numpy().tobytes()
        assert ta.tolist() == tb.tolist()
        for b in range(2):
            ol, _ = om.decode_token(pools[b], bt, pos, int(cur[b]))
            assert max_err_vs_row_max(la.cpu().numpy()[b], ol) <= DECODE_LOGIT_TOL
        cur = ta.astype(np.int32)
    # Malformed payloads: bad magic, wrong group, truncated, wrong element count, not INT4.
    good = bytearray(payloads[(0, _lib.W_O)])
    bad_magic = bytearray(good); bad_magic[0] ^= 1
    bad_group = bytearray(good); bad_group[8:12] = (16).to_bytes(4, "little")
    bad_prec = bytearray(good); bad_prec[12] = 2
    truncated = good[:-1]
    wrong_n = bytes(oracle.qio_encode(np.zeros(cfg.dim * cfg.dim // 2, np.float32), 32))
    h = _lib.handle(_lib.lib().glacier_cuda_model_create(C.byref(_lib.ModelConfigC(
        2, 256, 512, 8, 2, 64, 1000, 32, 1e-6, 1e6, 64, 1))))
    try:
        for pl in (bad_magic, bad_group, bad_prec, truncated, wrong_n):
            buf = np.frombuffer(bytes(pl), np.uint8)
            assert _lib.lib().glacier_cuda_model_load_qio(h, 0, _lib.W_O, buf.ctypes.data, buf.size) == _lib.EINVAL
    finally:
        _lib.lib().glacier_cuda_model_destroy(h)
    for s in (sa, sb):
        s.close()
    da.close()
    db.close()
