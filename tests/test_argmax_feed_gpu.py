# SPDX-License-Identifier: MIT
"""GPU: qh_argmax_feed (sample_argmax, slm/model.c:401-412, plus the device
feed of the next input) against numpy on rows with ties, NaNs and -inf,
for one and many rows and for vocabularies with and without float4 rows.
Two calls in a row on one scratch: the slice counters return to zero and
the position advances once per call."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _want(row):
    """First index of the strict maximum, scanning from element 0: a NaN at
    0 is never replaced, NaNs elsewhere never win."""
    if np.isnan(row[0]):
        return 0
    return int(np.argmax(np.where(np.isnan(row), -np.inf, row)))


@pytest.mark.parametrize("B,vocab", [(1, 151936), (3, 151936), (64, 151936), (5, 1001), (64, 4096)])
def test_argmax_feed_matches_first_strict_max(qh, cuda, B, vocab):
    torch = cuda
    L = qh.lib()
    rng = np.random.default_rng(B * 7 + vocab)
    logits = rng.standard_normal((B, vocab)).astype(np.float32)
    for r in range(B):
        k = r % 5
        if k == 1:  # a tie: the smaller index wins
            i, j = sorted(rng.choice(vocab, 2, replace=False))
            logits[r, i] = logits[r, j] = 9.0
        elif k == 2:  # NaNs away from 0 are never picked
            logits[r, rng.choice(vocab, 7, replace=False)] = np.nan
        elif k == 3 and r > 0:  # NaN at element 0: the pick is 0
            logits[r, 0] = np.nan
        elif k == 4:  # the maximum in the last element
            logits[r, -1] = 50.0
    if B > 2:
        logits[2, :] = -np.inf  # nothing beats element 0
    want = np.array([_want(logits[r]) for r in range(B)], np.int32)

    def P(t):
        return C.c_void_p(t.data_ptr())

    d_logits = torch.from_numpy(logits).cuda()
    nbytes = int(L.qh_argmax_feed_scratch_bytes(B, vocab))
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    stride = 8
    nxt = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    prompt = torch.zeros((B, stride), dtype=torch.int32, device="cuda")
    ctl = torch.tensor([2, 1, 0, 0], dtype=torch.int32, device="cuda")  # position 2, prompt of 1 token
    tokens = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    picks = torch.full((B, stride), -1, dtype=torch.int32, device="cuda")
    for call in range(2):
        qh.check(L.qh_argmax_feed(P(d_logits), B, vocab, P(scratch), P(nxt), P(prompt), stride, P(ctl), P(tokens),
                                  P(picks), None), "qh_argmax_feed")
        torch.cuda.synchronize()
        assert np.array_equal(nxt.cpu().numpy(), want), f"call {call}"
        assert np.array_equal(tokens.cpu().numpy(), want)
        assert np.array_equal(picks.cpu().numpy()[:, 2 + call], want)
        assert int(ctl[0]) == 3 + call
        # the B + 1 counters follow the partial maxima of at most 64 slices per row
        pmax = min(64, max(1, -(-vocab // 1024)))
        off = B * pmax * 8
        assert int(scratch[off:off + (B + 1) * 4].abs().sum()) == 0, "counters not returned to zero"
    assert L.qh_check_device_error(None) == 0
