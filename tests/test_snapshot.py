# SPDX-License-Identifier: MIT
"""GPU: device snapshot / restore of the decode state (qh_slm_snapshot,
qh_slm_restore) against the reference's slm_ctx_snapshot / slm_ctx_restore
(slm/model.c:1262-1371) on the same synthetic weights.

Schedule, per sequence: a prompt, snapshot, one continuation, restore, a
different continuation, restore again, the first continuation once more.
Bar: every logits vector bit-identical to the reference's (correctly
rounded expf/logf build), and the replayed continuation bit-identical to
its first run.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(qh, cuda):
    cfg = qh.host.slm_config(48, n_layers=4, vocab=4096)
    blob = qh.host.Blob(cfg, 0x5A9)
    return cfg, blob, blob.tensors()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def device_steps(slm, toks, pos0):
    return np.stack([slm.step(toks[:, i], pos0 + i, want_logits=True)[1] for i in range(toks.shape[1])], 1)


@pytest.mark.parametrize("B", [2, 12])
def test_snapshot_restore_matches_reference(qh, cuda, ref, model, B):
    from oracle.oracle import RefModel
    cfg, blob, tensors = model
    rng = np.random.default_rng(40 + B)
    n_p, n_c = 10, 8
    prompt = rng.integers(0, cfg.vocab, (B, n_p)).astype(np.int32)
    cont_a = rng.integers(0, cfg.vocab, (B, n_c)).astype(np.int32)
    cont_b = rng.integers(0, cfg.vocab, (B, n_c)).astype(np.int32)
    slm = qh.host.Slm(cfg, blob, B)
    slm.reset()
    device_steps(slm, prompt, 0)
    snap = slm.snapshot()
    assert snap.pos == n_p and snap.nbytes > 0
    la = device_steps(slm, cont_a, n_p)
    slm.restore(snap)
    lb = device_steps(slm, cont_b, n_p)
    slm.restore(snap)
    la2 = device_steps(slm, cont_a, n_p)
    snap.close()
    slm.close()
    assert np.array_equal(bits(la2), bits(la)), "replay after restore differs"
    for b in range(min(B, 2)):
        rm = RefModel(ref, cfg, tensors)
        for i in range(n_p):
            rm.step(int(prompt[b, i]), i)
        rs = rm.snapshot(n_p)
        ra = np.stack([rm.step(int(cont_a[b, i]), n_p + i, want_logits=True)[1] for i in range(n_c)])
        rm.restore(rs)
        rb = np.stack([rm.step(int(cont_b[b, i]), n_p + i, want_logits=True)[1] for i in range(n_c)])
        rm.free_snapshot(rs)
        rm.close()
        assert np.array_equal(bits(la[b]), bits(ra)), f"sequence {b}: first continuation differs"
        assert np.array_equal(bits(lb[b]), bits(rb)), f"sequence {b}: continuation after restore differs"


def test_restore_rejects_other_model(qh, cuda, model):
    cfg, blob, _ = model
    a, b = qh.host.Slm(cfg, blob, 1), qh.host.Slm(cfg, blob, 1)
    a.reset()
    a.step(np.array([5], np.int32), 0)
    snap = a.snapshot()
    with pytest.raises(qh.QHError):
        b.restore(snap)
    snap.close()
    a.close()
    b.close()


def test_snapshot_then_device_decode(qh, cuda, model):
    """A snapshot taken after qh_slm_prefill restores the device-driven
    greedy decode: the picks after restore equal the first run's."""
    cfg, blob, _ = model
    B = 3
    prompt = (np.arange(B * 12, dtype=np.int32).reshape(B, 12) * 97) % cfg.vocab
    slm = qh.host.Slm(cfg, blob, B)
    slm.prefill(prompt)
    snap = slm.snapshot()
    slm.advance(10)
    first = slm.picks(11, 10)
    slm.advance(5)
    slm.restore(snap)
    slm.advance(10)
    again = slm.picks(11, 10)
    snap.close()
    slm.close()
    assert np.array_equal(first, again)
