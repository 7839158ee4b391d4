"""The allocation-free greedy selection entry point, checked against the workspace one.

glacier_cuda_argmax_eligible_f32_noalloc serves callers that cannot allocate device memory
when they select tokens: a runtime that budgets all GPU memory when it admits requests, or a
plugin handed buffers but no allocator. It keeps its partial winners in a fixed 64 KiB
array inside the library instead of a caller workspace. These tests call it through the C ABI
twice in a row (the second call finds the first call's leftovers in that array) and require
exactly the tokens, statuses and result records of glacier_cuda_argmax_eligible_f32.

This file is named so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

EINVAL = -1
SCRATCH_BYTES = 65536  # GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES


def _lib():
    from glacier_b200._lib import lib
    return lib()


def _outputs(batch):
    from glacier_b200._lib import ArgmaxResult
    tokens = torch.full((batch,), -7, dtype=torch.int32, device="cuda")
    status = torch.full((batch,), -7, dtype=torch.int32, device="cuda")
    results = torch.zeros(batch * C.sizeof(ArgmaxResult), dtype=torch.uint8, device="cuda")
    return tokens, status, results


def _records(results):
    from glacier_b200._lib import ArgmaxResult
    raw = results.cpu().numpy().tobytes()
    n = len(raw) // C.sizeof(ArgmaxResult)
    recs = (ArgmaxResult * n).from_buffer_copy(raw)
    return [(r.value, r.index, r.valid, r.saw_nan) for r in recs]


def _with_workspace(logits, words):
    L = _lib()
    b, n = logits.shape
    ws_n = L.glacier_cuda_argmax_workspace(b, n)
    ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
    tokens, status, results = _outputs(b)
    wc = 0 if words is None else words.shape[1]
    rc = L.glacier_cuda_argmax_eligible_f32(logits.data_ptr(), b, n, None if words is None else words.data_ptr(),
                                            wc, tokens.data_ptr(), status.data_ptr(), results.data_ptr(),
                                            ws.data_ptr(), ws_n, None)
    assert rc == 0, L.glacier_cuda_last_error()
    torch.cuda.synchronize()
    return tokens.cpu().tolist(), status.cpu().tolist(), _records(results)


def _no_alloc(logits, words):
    L = _lib()
    b, n = logits.shape
    tokens, status, results = _outputs(b)
    wc = 0 if words is None else words.shape[1]
    rc = L.glacier_cuda_argmax_eligible_f32_noalloc(logits.data_ptr(), b, n,
                                                    None if words is None else words.data_ptr(), wc,
                                                    tokens.data_ptr(), status.data_ptr(), results.data_ptr(), None)
    assert rc == 0, L.glacier_cuda_last_error()
    torch.cuda.synchronize()
    return tokens.cpu().tolist(), status.cpu().tolist(), _records(results)


def _masked_case(seed, batch, n):
    """Random logits with random eligibility masks; a few planted ties and an eligible NaN."""
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal((batch, n), dtype=np.float32)
    words = rng.integers(0, 2**63, size=(batch, (n + 63) // 64), dtype=np.uint64)
    if n % 64:
        words[:, -1] &= np.uint64((1 << (n % 64)) - 1)
    lg[0, 7] = lg[0, n - 3] = 90.0
    words[0, 0] |= np.uint64(1 << 7)
    words[0, (n - 3) // 64] |= np.uint64(1 << ((n - 3) % 64))
    if batch > 2:
        lg[2, 11] = np.nan
        words[2, 0] |= np.uint64(1 << 11)
    return (torch.from_numpy(lg).cuda(), torch.from_numpy(words.view(np.int64)).cuda())


def test_no_alloc_matches_workspace_entry_on_two_calls_in_a_row():
    # First call: 64 lanes over a 152064-token vocabulary with masks (19 partials per row).
    lg1, w1 = _masked_case(1, 64, 152064)
    first = _no_alloc(lg1, w1)
    assert first == _with_workspace(lg1, w1)
    assert first[1][2] == -5 and first[0][2] == -1  # eligible NaN -> EligibleLogitNaN
    assert first[0][0] == 7  # tie resolves to the lowest index
    # Second call, smaller and unmasked: it must not be disturbed by the first call's leftovers.
    lg2 = torch.randn(5, 70000, device="cuda")
    lg2[3, 69999] = 1e30
    second = _no_alloc(lg2, None)
    assert second == _with_workspace(lg2, None)
    assert second[0][3] == 69999 and second[1] == [0] * 5
    # And a third call back at the first shape gives the first answer again.
    assert _no_alloc(lg1, w1) == first


def test_no_alloc_rejects_calls_beyond_its_fixed_scratch():
    L = _lib()
    n = 152064
    chunks = (n + 8191) // 8192
    batch = (SCRATCH_BYTES - 64) // (16 * chunks) + 1  # 216 rows: one more than fits
    lg = torch.zeros((batch, n), device="cuda")
    tokens, status, results = _outputs(batch)
    rc = L.glacier_cuda_argmax_eligible_f32_noalloc(lg.data_ptr(), batch, n, None, 0, tokens.data_ptr(),
                                                    status.data_ptr(), results.data_ptr(), None)
    assert rc == EINVAL
    assert b"fixed scratch" in L.glacier_cuda_last_error()
    torch.cuda.synchronize()
    assert tokens.cpu().tolist() == [-7] * batch  # nothing was written
    # One row fewer fits and agrees with the workspace entry point.
    lg = torch.randn((batch - 1, n), device="cuda")
    assert _no_alloc(lg, None) == _with_workspace(lg, None)
