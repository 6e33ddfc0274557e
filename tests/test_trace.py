# SPDX-License-Identifier: MIT
"""GPU: the device parity tracer (qh_slm_trace) against the reference's own
JSONL tracer (slm_trace_f32, slm/model.c:585-727) on the same synthetic
weights and token schedule.

Bar: every line the device writes is textually identical to the
reference's line of the same name (same fnv64 of the raw bytes, same head,
tail and sum), the device's names appear in the reference's order, and only
the intermediates the device never holds are missing.
"""
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# reference records of a Gated DeltaNet layer the device does not hold
NOT_ON_DEVICE = ("conv_raw", "Q_raw", "K_raw", "a_softplus", "g_in", "conv_silu")


def read(path):
    lines = open(path).read().splitlines()
    return [json.loads(l)["name"] for l in lines], {json.loads(l)["name"]: l for l in lines}


@pytest.mark.parametrize("B,seq", [(1, 0), (3, 1), (12, 7)])
def test_trace_matches_reference(qh, cuda, ref, tmp_path, B, seq):
    from oracle.oracle import RefModel
    cfg = qh.host.slm_config(32, n_layers=4, vocab=4096)
    blob = qh.host.Blob(cfg, 0x7A + B)
    rng = np.random.default_rng(B)
    prompt = rng.integers(0, cfg.vocab, (B, 6)).astype(np.int32)
    slm = qh.host.Slm(cfg, blob, B)
    slm.reset()
    for p in range(5):
        slm.step(prompt[:, p], p)
    dev_path = str(tmp_path / "device.jsonl")
    slm.trace(seq, dev_path)
    _, logits = slm.step(prompt[:, 5], 5, want_logits=True)
    # the step after the traced one runs from the graph again and agrees
    nxt = slm.step(np.full(B, 3, np.int32), 6)
    slm.close()
    rm = RefModel(ref, cfg, blob.tensors())
    for p in range(5):
        rm.step(int(prompt[seq, p]), p)
    ref_path = str(tmp_path / "ref.jsonl")
    rm.trace_step(ref_path, int(prompt[seq, 5]), 5)
    want_next = rm.step(3, 6)
    rm.close()
    dn, dl = read(dev_path)
    rn, rl = read(ref_path)
    missing = [n for n in rn if n not in dl]
    assert all(n.rsplit("-", 1)[0] in NOT_ON_DEVICE for n in missing), f"untraced: {missing}"
    assert len(dn) == len(rn) - len(NOT_ON_DEVICE) * sum(1 for n in rn if n.startswith("attn_qkv-"))
    assert [n for n in rn if n in dl] == dn, "record order differs"
    diff = [n for n in dn if dl[n] != rl[n]]
    assert not diff, f"records differ from the reference: {diff[:5]}"
    assert int(nxt[seq]) == want_next
    assert json.loads(dl["result_output"])["nbytes"] == 4 * cfg.vocab
    assert np.isfinite(logits).all()
