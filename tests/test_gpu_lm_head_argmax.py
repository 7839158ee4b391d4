"""The decode step's greedy selection against the semantics of argmaxEligible
(src/sampling.zig:55-107) -- logitless steps, masks, tail bits, NaN rows -- in both forms: the
argmax in the LM head GEMV's epilogue (4 lanes or fewer) and the tcgen05 GEMM's logits followed
by the two-pass argmax (more lanes).  And a position past the block table: context clamped to 0,
the bad-input word raised, the next step unharmed.

Decode parity against the oracle runs through tests/test_gpu_decode.py and test_gpu_configs.py.
"""
import numpy as np
import pytest

import oracle
from helpers import DECODE_LOGIT_TOL, max_err_vs_row_max

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _cfg():
    from glacier_b200.model import ModelConfig
    return ModelConfig(num_layers=2, dim=512, hidden=1024, num_heads=28, num_kv_heads=4, head_dim=128, vocab=2048)


def _session(model, lanes, max_pages=8, seed=1):
    from glacier_b200.model import DecodeSession, DeviceModel
    dm = DeviceModel(model, max_positions=max_pages * 16)
    sess = DecodeSession(dm, lanes, max_pages)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    sess.pages().normal_(generator=g)
    return dm, sess


@pytest.mark.parametrize("lanes", [3, 9])
def test_logitless_step_picks_the_argmax_of_the_logits_step(lanes):
    """Without a logits buffer the LM head writes no logits; the ids equal those of the same step
    with logits, which are the first maximum of each row."""
    from glacier_b200.model import SyntheticModel
    dm, sess = _session(SyntheticModel(_cfg(), seed=4), lanes)
    start = sess.pages().clone()
    toks, pos = list(range(5, 5 + lanes)), list(range(30, 30 + lanes))
    lg = torch.full((lanes, 2048), float("nan"), dtype=torch.float32, device="cuda")
    with_logits = sess.step(tokens=toks, positions=pos, logits=lg).cpu().tolist()
    rows = lg.cpu().numpy()
    assert with_logits == [int(np.argmax(r)) for r in rows]
    sess.pages().copy_(start)
    logitless = sess.step(tokens=toks, positions=pos).cpu().tolist()
    assert logitless == with_logits and sess.status.cpu().tolist() == [0] * lanes
    sess.close()
    dm.close()


@pytest.mark.parametrize("lanes", [4, 12])
def test_argmax_epilogue_masks_tail_bits_and_empty_masks(lanes):
    """Lane i follows pattern i % 4.  0: tokens 192..207 only; 1: every token; 2: token 0 only;
    3: no bit set (InvalidEligibleMask).  Then a vocabulary that is not a multiple of 64: a bit
    past it (InvalidEligibleMask) or the last token alone."""
    from glacier_b200 import _lib
    from glacier_b200.model import SyntheticModel
    cfg = _cfg()
    dm, sess = _session(SyntheticModel(cfg, seed=6), lanes)
    words = np.zeros((lanes, cfg.vocab // 64), np.uint64)
    for b in range(lanes):
        if b % 4 == 0:
            words[b, 3] = 0xFFFF
        elif b % 4 == 1:
            words[b, :] = np.uint64(0xFFFFFFFFFFFFFFFF)
        elif b % 4 == 2:
            words[b, 0] = 1
    lg = torch.empty((lanes, cfg.vocab), dtype=torch.float32, device="cuda")
    elig = torch.from_numpy(words.view(np.int64)).cuda()
    toks, pos = list(range(1, 1 + lanes)), list(range(20, 20 + lanes))
    out = sess.step(tokens=toks, positions=pos, eligible=elig, logits=lg).cpu().tolist()
    rows = lg.cpu().numpy()
    st = sess.status.cpu().tolist()
    for b in range(lanes):
        if b % 4 == 0:
            assert out[b] == 192 + int(np.argmax(rows[b, 192:208])) and st[b] == 0, b
        elif b % 4 == 1:
            assert out[b] == int(np.argmax(rows[b])) and st[b] == 0, b
        elif b % 4 == 2:
            assert out[b] == 0 and st[b] == 0, b
        else:
            assert out[b] == -1 and st[b] == _lib.EMASK, b
    sess.close()
    dm.close()
    from glacier_b200.model import ModelConfig
    cfg2 = ModelConfig(num_layers=1, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)
    dm, sess = _session(SyntheticModel(cfg2, seed=2), lanes)
    w2 = np.zeros((lanes, -(-cfg2.vocab // 64)), np.uint64)
    for b in range(lanes):
        if b % 2 == 0:
            w2[b, -1] = np.uint64(1) << np.uint64(1000 % 64)  # bit 1000: past the vocabulary
            w2[b, 0] = 1
        else:
            w2[b, -1] = np.uint64(1) << np.uint64(1000 % 64 - 1)  # bit 999: the last token
    out = sess.step(tokens=list(range(lanes)), positions=list(range(3, 3 + lanes)),
                    eligible=torch.from_numpy(w2.view(np.int64)).cuda())
    assert sess.status.cpu().tolist() == [_lib.EMASK if b % 2 == 0 else 0 for b in range(lanes)]
    assert out.cpu().tolist() == [-1 if b % 2 == 0 else 999 for b in range(lanes)]
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    sess.close()
    dm.close()


@pytest.mark.parametrize("lanes", [2, 8])
def test_argmax_epilogue_reports_an_eligible_nan_row(lanes):
    """An LM-head row whose scales are NaN gives a NaN logit: EligibleLogitNaN for every lane
    unless the mask leaves that token out."""
    from glacier_b200 import _lib
    from glacier_b200.model import SyntheticModel
    cfg = _cfg()
    m = SyntheticModel(cfg, seed=8)
    packed, scales = m.lm_head
    scales = scales.copy().reshape(cfg.vocab, -1)
    scales[777] = np.nan
    m.lm_head = (packed, scales.ravel())
    dm, sess = _session(m, lanes)
    toks, pos = list(range(3, 3 + lanes)), list(range(10, 10 + lanes))
    out = sess.step(tokens=toks, positions=pos).cpu().tolist()
    assert sess.status.cpu().tolist() == [_lib.ENAN] * lanes and out == [-1] * lanes
    words = np.full((lanes, cfg.vocab // 64), np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64)
    words[:, 777 // 64] &= ~(np.uint64(1) << np.uint64(777 % 64))
    lg = torch.empty((lanes, cfg.vocab), dtype=torch.float32, device="cuda")
    out = sess.step(tokens=toks, positions=pos, eligible=torch.from_numpy(words.view(np.int64)).cuda(),
                    logits=lg).cpu().tolist()
    rows = lg.cpu().numpy()
    assert np.isnan(rows[:, 777]).all()
    rows[:, 777] = -np.inf
    assert sess.status.cpu().tolist() == [0] * lanes and out == [int(np.argmax(r)) for r in rows]
    sess.close()
    dm.close()


def test_bad_position_raises_the_input_word_and_the_next_step_matches_the_oracle():
    """A position past the block table: no KV write, context 0 for that lane, device status 2
    (bad input); the following valid step of the other lane still matches the oracle."""
    from glacier_b200 import _lib
    from glacier_b200.model import ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=2, dim=256, hidden=512, num_heads=8, num_kv_heads=2, head_dim=64, vocab=1000)
    m = SyntheticModel(cfg, seed=3)
    max_pages = 4
    dm, sess = _session(m, 2, max_pages=max_pages)
    sess.pages().zero_()
    om = oracle.OracleModel(m, rope_positions=max_pages * 16, threads=2)
    pool = np.zeros(max_pages * om.page_floats(), np.float32)
    bt = np.arange(max_pages, dtype=np.int32)
    sess.step(tokens=[1, 2], positions=[0, max_pages * 16 + 5])
    torch.cuda.synchronize()
    assert _lib.lib().glacier_cuda_device_status(1) == 2
    om.decode_token(pool, bt, 0, 1)  # lane 0's first position, as the device appended it
    lg = torch.empty((2, cfg.vocab), dtype=torch.float32, device="cuda")
    sess.step(tokens=[9, 2], positions=[1, 0], logits=lg)
    ol, _ = om.decode_token(pool, bt, 1, 9)
    assert max_err_vs_row_max(lg.cpu().numpy()[0], ol) <= DECODE_LOGIT_TOL
    assert _lib.lib().glacier_cuda_device_status(1) == 0
    sess.close()
    dm.close()
