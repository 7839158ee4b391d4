"""Decode parity at the shapes the bench measures (3 and 5) vs the CPU oracle.

Each case keeps the configuration's full geometry -- layer widths, head layout, the real
vocabulary -- and its context lengths; only the number of decoded tokens is trimmed so the
oracle (the reference's portable FP32 path restated in C) finishes in seconds.  Context that
a lane has already seen is random FP32 K/V rows written into its pages on both sides (decode
cost and arithmetic depend only on the rows, not on how they were produced); the positions a
case decodes are appended by the kernels themselves and by the oracle's own kv_append.

Bounds are the decode contract of tests/test_gpu_decode.py: logits within DECODE_LOGIT_TOL of
the row's largest |logit|, greedy ids exact except at documented near-ties (oracle top-2 gap
below 1e-3 * max(1, |top1|)), after which a lane is no longer compared.
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


def _threads() -> int:
    import os
    try:
        return max(1, min(16, len(os.sched_getaffinity(0))))
    except AttributeError:
        return 8


class _Lanes:
    """Host pools of the lanes the oracle follows, mirrored into the session's pages."""

    def __init__(self, sess, om, checked, ctxs, seed):
        self.sess, self.om = sess, om
        self.pf = om.page_floats()
        self.bt = np.arange(sess.max_pages, dtype=np.int32)
        pages = sess.pages()
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        for i in range(0, pages.shape[0], 256):
            pages[i:i + 256].normal_(generator=g)
        rng = np.random.default_rng(seed)
        self.pools = {}
        for b in checked:
            # Only the rows before the lane's context matter; the rest is overwritten or masked.
            used = -(-int(ctxs[b]) // 16)
            pool = np.zeros(sess.max_pages * self.pf, np.float32)
            pool[:used * self.pf] = rng.standard_normal(used * self.pf, dtype=np.float32)
            pages[b * sess.max_pages:b * sess.max_pages + used].copy_(
                torch.from_numpy(pool[:used * self.pf].reshape(used, self.pf)))
            self.pools[b] = pool
        torch.cuda.synchronize()

    def oracle_logits(self, b, pos, token):
        ol, _ = self.om.decode_token(self.pools[b], self.bt, int(pos), int(token))
        return ol


def _decode_and_compare(cfg, lanes, ctxs, checked, steps, seed, layers=None, reserve=None):
    from glacier_b200.model import DecodeSession, DeviceModel, SyntheticModel
    m = SyntheticModel(cfg, seed=seed, layers=layers)
    max_pages = -(-(int(max(ctxs)) + steps + 1) // 16)
    dm = DeviceModel(m, max_positions=max_pages * 16)
    sess = DecodeSession(dm, lanes, max_pages, reserve_lanes=reserve)
    om = oracle.OracleModel(m, rope_positions=max_pages * 16, threads=_threads())
    kv = _Lanes(sess, om, checked, ctxs, seed)
    rng = np.random.default_rng(seed + 1)
    cur = rng.integers(0, cfg.vocab, size=lanes).astype(np.int32)
    pos = np.asarray(ctxs, np.int32).copy()
    logits = torch.empty((lanes, cfg.vocab), dtype=torch.float32, device="cuda")
    live = {b: True for b in checked}
    compared = 0
    for _ in range(steps):
        out = sess.step(tokens=cur, positions=pos, logits=logits).cpu().numpy()
        assert sess.status.cpu().numpy().tolist() == [0] * lanes
        gl = logits.cpu().numpy()
        for b in checked:
            ol = kv.oracle_logits(b, pos[b], cur[b])
            if not live[b]:
                continue
            assert max_err_vs_row_max(gl[b], ol) <= DECODE_LOGIT_TOL, (b, int(pos[b]))
            if out[b] != oracle.argmax(ol):
                assert near_tie(ol), (b, int(pos[b]), int(out[b]), oracle.argmax(ol))
                live[b] = False
            else:
                compared += 1
        cur = out.astype(np.int32)
        pos += 1
    from glacier_b200 import _lib
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    sess.close()
    dm.close()
    return compared


def test_config2_05b_full_model_prefill_then_batch1_decode():
    """Config 2 at its full shape: 24 layers, D 896, FFN 4864, 14/2 heads of 64, vocab 151936.
    The lane's first 496 positions are random K/V rows; a 16-token prompt chunk then runs through
    glacier_cuda_prefill (positions 496..511, context 512) on a 4-lane reservation, and greedy
    batch-1 decode follows from context 512 on a one-lane reservation."""
    from glacier_b200.model import PRESETS, DecodeSession, DeviceModel, SyntheticModel
    cfg = PRESETS["qwen2.5-0.5b"]
    seed, ctx0, prompt_len, steps = 21, 496, 16, 12
    m = SyntheticModel(cfg, seed=seed)
    max_pages = -(-(ctx0 + prompt_len + steps + 1) // 16)
    dm = DeviceModel(m, max_positions=max_pages * 16)
    sess = DecodeSession(dm, 1, max_pages, reserve_lanes=4)
    om = oracle.OracleModel(m, rope_positions=max_pages * 16, threads=_threads())
    kv = _Lanes(sess, om, [0], [ctx0], seed)
    rng = np.random.default_rng(seed + 1)
    prompt = rng.integers(0, cfg.vocab, size=prompt_len).astype(np.int32)
    for i, t in enumerate(prompt):
        ol = kv.oracle_logits(0, ctx0 + i, t)
    lg = torch.empty(cfg.vocab, dtype=torch.float32, device="cuda")
    tok = int(sess.prefill(prompt, start=ctx0, logits=lg).cpu()[0])
    assert int(sess.last_status.cpu()[0]) == 0
    assert max_err_vs_row_max(lg.cpu().numpy(), ol) <= DECODE_LOGIT_TOL
    # Decode on a one-lane reservation (the bench's batch-1 path).
    from glacier_b200 import _lib
    _lib.call("glacier_cuda_model_reserve", dm.h, 1, max_pages)
    compared = 0
    pos = ctx0 + prompt_len
    step_lg = torch.empty((1, cfg.vocab), dtype=torch.float32, device="cuda")
    for i in range(steps + 1):
        ref = oracle.argmax(ol)
        if tok != ref:
            assert near_tie(ol), (pos, tok, ref)
            break
        compared += 1
        if i == steps:
            break
        out = int(sess.step(tokens=[tok], positions=[pos], logits=step_lg).cpu()[0])
        assert int(sess.status.cpu()[0]) == 0
        ol = kv.oracle_logits(0, pos, tok)
        assert max_err_vs_row_max(step_lg.cpu().numpy()[0], ol) <= DECODE_LOGIT_TOL, pos
        tok, pos = out, pos + 1
    from glacier_b200 import _lib
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    sess.close()
    dm.close()
    assert compared >= 6


def test_config3_15b_full_model_8_lanes():
    """Config 3 at its full shape: 28 layers, D 1536, FFN 8960, 12/2 heads of 128, vocab 151936,
    8 lanes (the tcgen05 GEMM path) at contexts spread over [128, 2048] (both ends included)."""
    from glacier_b200.model import PRESETS
    cfg = PRESETS["qwen2.5-1.5b"]
    rng = np.random.default_rng(33)
    ctxs = np.concatenate([[128, 2048], rng.integers(128, 2049, size=6)]).astype(np.int32)
    assert _decode_and_compare(cfg, 8, ctxs, list(range(8)), steps=3, seed=33) >= 16


def test_config5_7b_64_lanes_long_contexts():
    """Config 5's decode at 64 lanes on the tcgen05 GEMM: the full 7B layer widths (D 3584, FFN
    18944, 28/4 heads of 128) in two layers, the real 152064-token LM head, and lanes at
    contexts 4096, 4097, 4351 and 4352 (past the reference's 4096 cap, which the oracle lifts)
    beside lanes drawn from [256, 4096].  The oracle follows eight of the lanes."""
    from glacier_b200.model import PRESETS
    cfg = PRESETS["qwen2.5-7b"]
    rng = np.random.default_rng(55)
    ctxs = rng.integers(256, 4097, size=64).astype(np.int32)
    ctxs[:4] = [4096, 4097, 4351, 4352 - 2]
    checked = [0, 1, 2, 3, 17, 40, 63, 5]
    assert _decode_and_compare(cfg, 64, ctxs, checked, steps=2, seed=55, layers=2) >= 12
