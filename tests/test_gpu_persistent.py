"""The persistent one-lane decode step (one cooperative kernel per step) vs the CPU oracle and
vs the multi-kernel step it replaces.

Bounds are the decode contract of tests/test_gpu_decode.py: logits within DECODE_LOGIT_TOL of
the row's largest |logit|, greedy ids exact except at near-ties.
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


def _session(cfg, ctx, steps, seed):
    from glacier_b200 import _lib
    from glacier_b200.model import DecodeSession, DeviceModel, SyntheticModel
    m = SyntheticModel(cfg, seed=seed)
    max_pages = -(-(ctx + steps + 1) // 16)
    dm = DeviceModel(m, max_positions=max_pages * 16)
    sess = DecodeSession(dm, 1, max_pages)
    assert _lib.lib().glacier_cuda_model_persistent(dm.h, 1) == 1
    om = oracle.OracleModel(m, rope_positions=max_pages * 16, threads=8)
    pf = om.page_floats()
    rng = np.random.default_rng(seed)
    pool = np.zeros(max_pages * pf, np.float32)
    used = -(-ctx // 16)
    pool[:used * pf] = rng.standard_normal(used * pf, dtype=np.float32)
    sess.pages().copy_(torch.from_numpy(pool.reshape(max_pages, pf)))
    return m, dm, sess, om, pool


@pytest.mark.parametrize("geom,ctx", [
    ("7b", 5),      # one 16-position chunk per kv head, the new position in it
    ("7b", 1183),   # the bench's batch-1 context: several chunks per kv head, merged by the last CTA
    ("7b", 4350),   # past the reference's 4096 cap
    ("05b", 512),   # head dim 64, 14 / 2 heads
    ("small", 40),  # 8 / 2 heads of 64, short rows
])
def test_persistent_step_matches_oracle(geom, ctx):
    from glacier_b200.model import ModelConfig
    cfg = {"7b": ModelConfig(2, 3584, 18944, 28, 4, 128, 4096),
           "05b": ModelConfig(3, 896, 4864, 14, 2, 64, 3000),
           "small": ModelConfig(2, 256, 512, 8, 2, 64, 1000)}[geom]
    steps = 4
    m, dm, sess, om, pool = _session(cfg, ctx, steps, seed=ctx + cfg.dim)
    bt = np.arange(sess.max_pages, dtype=np.int32)
    logits = torch.empty((1, cfg.vocab), dtype=torch.float32, device="cuda")
    tok, pos, compared = 7, ctx, 0
    for _ in range(steps):
        out = int(sess.step(tokens=[tok], positions=[pos], logits=logits).cpu()[0])
        assert int(sess.status.cpu()[0]) == 0
        ol, _ = om.decode_token(pool, bt, pos, tok)
        assert max_err_vs_row_max(logits.cpu().numpy()[0], ol) <= DECODE_LOGIT_TOL, pos
        ref = oracle.argmax(ol)
        if out != ref:
            assert near_tie(ol), (pos, out, ref)
            break
        compared += 1
        tok, pos = out, pos + 1
    from glacier_b200 import _lib
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    sess.close()
    dm.close()
    assert compared >= 2


def test_persistent_and_multi_kernel_steps_agree():
    """The same greedy steps from the same KV state through both step forms: identical ids,
    logits equal to rounding, and the KV pages they append equal to rounding."""
    from glacier_b200 import _lib
    from glacier_b200.model import ModelConfig
    cfg = ModelConfig(2, 3584, 18944, 28, 4, 128, 4096)
    m, dm, sess, om, pool = _session(cfg, 700, 6, seed=3)
    start = sess.pages().clone()
    runs = []
    for enable in (1, 0):
        _lib.lib().glacier_cuda_model_persistent(dm.h, enable)
        sess.pages().copy_(start)
        lg = torch.empty((1, cfg.vocab), dtype=torch.float32, device="cuda")
        toks, logs = [], []
        tok, pos = 11, 700
        for _ in range(6):
            tok = int(sess.step(tokens=[tok], positions=[pos], logits=lg).cpu()[0])
            toks.append(tok)
            logs.append(lg.cpu().numpy()[0].copy())
            pos += 1
        runs.append((toks, logs, sess.pages().clone()))
    assert runs[0][0] == runs[1][0]
    for a, b in zip(runs[0][1], runs[1][1]):
        assert max_err_vs_row_max(a, b) <= DECODE_LOGIT_TOL
    pa, pb = runs[0][2], runs[1][2]
    assert float((pa - pb).abs().max()) <= 1e-5 * float(pb.abs().max())
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    sess.close()
    dm.close()


def test_persistent_step_eligible_mask_graph_replay_and_profile():
    """Eligibility masks reach the argmax after the persistent kernel; a CUDA graph of the
    greedy step replays it; profiling files its phases under the replaced kernel classes."""
    import ctypes as C
    from glacier_b200 import _lib
    from glacier_b200.model import ModelConfig
    cfg = ModelConfig(2, 512, 1024, 28, 4, 128, 2048)
    m, dm, sess, om, pool = _session(cfg, 100, 8, seed=9)
    lg = torch.empty((1, cfg.vocab), dtype=torch.float32, device="cuda")
    words = np.zeros((1, cfg.vocab // 64), np.uint64)
    words[0, 3] = 0xFFFF  # tokens 192..207 only
    elig = torch.from_numpy(words.view(np.int64)).cuda()
    out = int(sess.step(tokens=[5], positions=[100], eligible=elig, logits=lg).cpu()[0])
    row = lg.cpu().numpy()[0]
    assert out == 192 + int(np.argmax(row[192:208]))
    # Graph replay: same ids as stream steps from the same state.
    sess.pages().copy_(torch.from_numpy(pool.reshape(sess.max_pages, -1)))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        sess.tokens.fill_(5)
        sess.positions.fill_(100)
        plain = []
        for _ in range(3):
            o = sess.step(stream=s)
            sess.tokens.copy_(o)
            sess.positions.add_(1)
            plain.append(int(o.cpu()[0]))
        sess.pages().copy_(torch.from_numpy(pool.reshape(sess.max_pages, -1)))
        sess.tokens.fill_(5)
        sess.positions.fill_(100)
        sess.capture_greedy_step(stream=s)
        sess.pages().copy_(torch.from_numpy(pool.reshape(sess.max_pages, -1)))
        sess.tokens.fill_(5)
        sess.positions.fill_(100)
        replayed = [int(sess.replay_greedy_step().cpu()[0]) for _ in range(3)]
    torch.cuda.synchronize()
    assert replayed == plain
    _lib.call("glacier_cuda_model_profile", dm.h, 1)
    for _ in range(2):
        sess.step(tokens=[5], positions=[100])
    _lib.call("glacier_cuda_model_profile", dm.h, 0)
    n = 12
    ms, regions = (C.c_double * n)(), (C.c_uint64 * n)()
    _lib.call("glacier_cuda_model_profile_read", dm.h, ms, regions, n)
    per = [r // 2 for r in regions]
    assert per[2] == per[4] == per[6] == per[7] == per[9] == cfg.num_layers  # qkv, attn, o, gate_up, down
    assert per[10] == per[11] == 1 and all(ms[k] > 0 for k in (2, 4, 6, 7, 9, 10, 11))
    sess.close()
    dm.close()


def test_persistent_step_rejects_a_bad_position_and_recovers():
    """A position past the block table ends the launch at once with the device status word set
    (no barrier waits); the next valid step runs normally."""
    from glacier_b200 import _lib
    from glacier_b200.model import ModelConfig
    cfg = ModelConfig(1, 256, 512, 8, 2, 64, 1000)
    m, dm, sess, om, pool = _session(cfg, 10, 2, seed=4)
    out = sess.step(tokens=[1], positions=[sess.max_pages * 16 + 3])
    assert int(out.cpu()[0]) == -1 and int(sess.status.cpu()[0]) == _lib.EINVAL
    assert _lib.lib().glacier_cuda_device_status(1) == 2
    lg = torch.empty((1, cfg.vocab), dtype=torch.float32, device="cuda")
    out = int(sess.step(tokens=[1], positions=[10], logits=lg).cpu()[0])
    ol, _ = om.decode_token(pool, np.arange(sess.max_pages, dtype=np.int32), 10, 1)
    assert max_err_vs_row_max(lg.cpu().numpy()[0], ol) <= DECODE_LOGIT_TOL
    assert out == oracle.argmax(ol) or near_tie(ol)
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    sess.close()
    dm.close()
