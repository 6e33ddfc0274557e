# SPDX-License-Identifier: MIT
"""GPU: the chunked Gated DeltaNet prefill (qh_gdn_chunk_prep, qh_gdn_chunked,
QH_PREFILL_CHUNKED) against the reference's batched prompt path.

1. qh_gdn_chunked against the oracle's chunked step (orc_chunked_step,
   itself pinned bit-exact to the reference's chunked_ssm_step_f32 by
   tests/test_chunked_oracle.py), in slm_forward_ssm_batch's 64-token chunk
   loop: outputs and carried state bit-identical, ragged chunks included.
2. qh_gdn_chunk_prep against a float64-checked restatement of
   slm/qwen.c:652-715 (conv ring, SiLU, L2 norms, beta, g_log).
3. The model with QH_PREFILL_CHUNKED against the reference's own
   slm_forward_batch (the LLM_USE_FORWARD_BATCH prefill, slm/qwen.c:1018)
   followed by slm_forward_step: greedy picks and every logit vector
   bit-identical (the stock build: the device's expf/logf are the host library's).
"""
import ctypes as C

import numpy as np
import pytest

from tests.chunked_cases import chunk_inputs

pytestmark = pytest.mark.gpu

HD = 128


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def pack(n_seq, heads, n_tok, seed):
    """Rows of qkv [n_seq*n_tok][3*heads*HD], beta, g_log [rows][heads] and
    state [n_seq][heads][HD][HD] from per-(sequence, head) chunk inputs."""
    kdim = heads * HD
    qkv = np.zeros((n_seq * n_tok, 3 * kdim), np.float32)
    beta = np.zeros((n_seq * n_tok, heads), np.float32)
    glog = np.zeros_like(beta)
    state = np.zeros((n_seq, heads, HD, HD), np.float32)
    per = {}
    for s in range(n_seq):
        for h in range(heads):
            q, k, v, g, b, st = chunk_inputs(n_tok, HD, seed + 31 * s + h)
            rows = slice(s * n_tok, (s + 1) * n_tok)
            qkv[rows, h * HD:(h + 1) * HD] = q
            qkv[rows, kdim + h * HD:kdim + (h + 1) * HD] = k
            qkv[rows, 2 * kdim + h * HD:2 * kdim + (h + 1) * HD] = v
            beta[rows, h], glog[rows, h] = b, g
            state[s, h] = st
            per[s, h] = (q, k, v, g, b, st)
    return qkv, beta, glog, state, per


def run_chunked(qh, qkv, beta, glog, state, n_seq, n_tok, heads, splits=None):
    """qh_gdn_chunked over the rows, optionally as several launches of
    `splits` tokens each (state carried between them on the device)."""
    h = qh.host
    kdim = heads * HD
    d_state = h.to_device(state)
    out = np.empty((n_seq * n_tok, kdim), np.float32)
    splits = splits or [n_tok]
    t0 = 0
    for cn in splits:
        sl = lambda a: np.ascontiguousarray(a.reshape(n_seq, n_tok, -1)[:, t0:t0 + cn].reshape(n_seq * cn, -1))
        d_qkv, d_b, d_g = h.to_device(sl(qkv)), h.to_device(sl(beta)), h.to_device(sl(glog))
        d_out = h.to_device(np.zeros((n_seq * cn, kdim), np.float32))
        qh.check(qh.lib().qh_gdn_chunked(h.dptr(d_qkv), h.dptr(d_b), h.dptr(d_g), h.dptr(d_state), n_seq, cn, heads,
                                         HD, h.dptr(d_out), h.stream_handle()), "qh_gdn_chunked")
        qh.check(qh.lib().qh_check_device_error(None), "device error word")
        out.reshape(n_seq, n_tok, kdim)[:, t0:t0 + cn] = d_out.cpu().numpy().reshape(n_seq, cn, kdim)
        t0 += cn
    return out, d_state.cpu().numpy()


@pytest.mark.parametrize("n_seq,heads,n_tok,splits", [
    (1, 1, 1, None), (2, 3, 37, None), (1, 2, 64, None), (2, 2, 130, None), (3, 1, 200, [64, 128, 8]),
])
def test_chunked_kernel_matches_oracle(qh, cuda, oracle, n_seq, heads, n_tok, splits):
    qkv, beta, glog, state, per = pack(n_seq, heads, n_tok, 500 + n_tok)
    out, st = run_chunked(qh, qkv, beta, glog, state, n_seq, n_tok, heads, splits)
    for (s, h), (q, k, v, g, b, s0) in per.items():
        s_want = s0.copy()
        want = oracle.chunked_prefill(q, k, v, g, b, s_want)
        got = out[s * n_tok:(s + 1) * n_tok, h * HD:(h + 1) * HD]
        assert np.array_equal(bits(got), bits(want)), f"outputs of sequence {s} head {h} differ from the oracle"
        assert np.array_equal(bits(st[s, h]), bits(s_want)), f"state of sequence {s} head {h} differs"


def test_chunked_kernel_rejects_bad_arguments(qh, cuda):
    assert qh.lib().qh_gdn_chunked(None, None, None, None, 1, 1, 1, HD, None, None) != 0
    h = qh.host
    x = h.to_device(np.zeros(8 * 3 * HD, np.float32))
    assert qh.lib().qh_gdn_chunked(h.dptr(x), h.dptr(x), h.dptr(x), h.dptr(x), 1, 1, 1, 64, h.dptr(x), None) != 0


def test_chunk_prep_matches_restatement(qh, cuda):
    """Conv over the ring + the chunk's rows, SiLU, L2 norms (Q also
    scaled by 1/sqrt(hd)), beta and g_log (slm/qwen.c:652-715), ring left for
    the next chunk; float64 check within float rounding."""
    h = qh.host
    rng = np.random.default_rng(9)
    n_seq, heads, n_tok, kk, pos0 = 2, 2, 11, 4, 5
    kdim = heads * HD
    cd = 3 * kdim
    qkv = rng.standard_normal((n_seq * n_tok, cd)).astype(np.float32)
    ring = rng.standard_normal((n_seq, kk, cd)).astype(np.float32)
    conv_w = (rng.standard_normal(cd * kk) * 0.3).astype(np.float32)
    b = rng.standard_normal((n_seq * n_tok, heads)).astype(np.float32)
    a = rng.standard_normal((n_seq * n_tok, heads)).astype(np.float32)
    a[0, 0] = 25.0  # softplus above 20 is the identity
    dt = rng.standard_normal(heads).astype(np.float32)
    ssm_a = -np.exp(rng.normal(0, 0.02, heads)).astype(np.float32)
    d = [h.to_device(x) for x in (qkv, ring, conv_w, b, a, dt, ssm_a, np.array([pos0, 0, 0, 0], np.int32))]
    qh.check(qh.lib().qh_gdn_chunk_prep(*[h.dptr(x) for x in d[:7]], n_seq, n_tok, heads, HD, kk, h.dptr(d[7]),
                                        h.stream_handle()), "qh_gdn_chunk_prep")
    got_qkv, got_ring, got_b, got_a = (d[i].cpu().numpy() for i in (0, 1, 3, 4))
    f32 = np.float32
    w = conv_w.reshape(cd, kk)
    for s in range(n_seq):
        # history: positions pos0-3 .. pos0-1 live in slots (pos0+1+k) % kk
        hist = [ring[s, (pos0 + 1 + k) % kk] for k in range(kk - 1)]
        for j in range(n_tok):
            r = s * n_tok + j
            win = hist[-(kk - 1):] + [qkv[r]]
            conv = np.zeros(cd, f32)
            for k in range(kk):  # float sums in tap order, as the reference
                conv = (conv + (win[k] * w[:, k]).astype(f32)).astype(f32)
            hist.append(qkv[r])
            c64 = conv.astype(np.float64)
            mixed = c64 / (1.0 + np.exp(-c64))
            for hh in range(heads):
                sl = slice(hh * HD, (hh + 1) * HD)
                qv, kv, vv = mixed[sl], mixed[kdim:][sl], mixed[2 * kdim:][sl]
                want = np.concatenate([qv / max(np.linalg.norm(qv), 1e-6) / np.sqrt(HD),
                                       kv / max(np.linalg.norm(kv), 1e-6), vv])
                got = np.concatenate([got_qkv[r, sl], got_qkv[r, kdim:][sl], got_qkv[r, 2 * kdim:][sl]])
                np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7)
                av = f32(a[r, hh] + dt[hh])
                if av > 20:
                    sp = av
                else:
                    sp = f32(np.log(np.float64(f32(f32(1.0) + f32(np.exp(np.float64(av)))))))
                np.testing.assert_allclose(got_b[r, hh], 1 / (1 + np.exp(-np.float64(b[r, hh]))), rtol=1e-6)
                np.testing.assert_allclose(got_a[r, hh], f32(ssm_a[hh] * sp), rtol=1e-6)
        last = pos0 + n_tok - 1
        for k in range(kk - 1):
            p = last - (kk - 2) + k
            assert np.array_equal(got_ring[s, p % kk], qkv[s * n_tok + (p - pos0)]), "ring slot not left raw"


def ref_batch_then_steps(ref, cfg, tensors, prompt, n_new):
    """slm_forward_batch over prompt[:-1], then greedy slm_forward_step from
    the last prompt token: picks and logits of every step."""
    from oracle.oracle import RefModel
    rm = RefModel(ref, cfg, tensors)
    n = len(prompt)
    rm.forward_batch(prompt[:-1], 0)
    picks, logits = [], []
    tok = prompt[-1]
    for pos in range(n - 1, n - 1 + n_new + 1):
        a, lg = rm.step(tok, pos, want_logits=True)
        picks.append(a)
        logits.append(lg)
        tok = a
    rm.close()
    return np.array(picks), logits


def chunked_device_run(qh, cfg, blob, prompts, n_new, chunk=0):
    B, n = prompts.shape
    slm = qh.host.Slm(cfg, blob, B)
    slm.prefill(prompts, chunk, mode=qh.PREFILL_CHUNKED)
    slm.advance(n_new)
    got = slm.picks(n - 1, n_new)
    _, lg = slm.step(got[:, -1], n - 1 + n_new, want_logits=True)
    slm.close()
    return got, lg


@pytest.fixture(scope="module")
def small200(qh, cuda):
    cfg = qh.host.slm_config(200, n_layers=4, vocab=4096)
    blob = qh.host.Blob(cfg, 0x51A12)
    return cfg, blob, blob.tensors()


@pytest.mark.parametrize("B,n_prompt,chunk", [(1, 13, 0), (3, 150, 0), (2, 150, 5), (1, 66, 64)])
def test_chunked_prefill_matches_reference_forward_batch(qh, cuda, ref, small200, B, n_prompt, chunk):
    cfg, blob, tensors = small200
    n_new = 6
    rng = np.random.default_rng(60 + n_prompt + B)
    prompts = rng.integers(0, cfg.vocab, (B, n_prompt)).astype(np.int32)
    got, lg = chunked_device_run(qh, cfg, blob, prompts, n_new, chunk)
    for b in range(B):
        want, wl = ref_batch_then_steps(ref, cfg, tensors, prompts[b], n_new)
        assert np.array_equal(got[b], want[:n_new]), f"seq {b}: greedy picks after the chunked prefill differ"
        assert np.array_equal(bits(lg[b]), bits(wl[n_new])), f"seq {b}: logits after the chunked prefill differ"


def test_chunked_prefill_differs_from_stepwise(qh, cuda, small200):
    """The two prefill modes are different arithmetic (the reference's own
    paths disagree in the last bits): guards against the mode being ignored."""
    cfg, blob, _ = small200
    rng = np.random.default_rng(77)
    prompts = rng.integers(0, cfg.vocab, (1, 70)).astype(np.int32)
    _, lc = chunked_device_run(qh, cfg, blob, prompts, 2)
    slm = qh.host.Slm(cfg, blob, 1)
    slm.prefill(prompts)
    slm.advance(2)
    got = slm.picks(69, 2)
    _, ls = slm.step(got[:, -1], 71, want_logits=True)
    slm.close()
    assert not np.array_equal(bits(lc), bits(ls))


def test_chunked_prefill_full_model(qh, cuda, ref):
    """BASELINE config-4 shape (24 layers, vocab 151936), 64-token prompt:
    the chunked prefill then 8 greedy steps, logits bit-identical to the
    reference's slm_forward_batch + slm_forward_step."""
    cfg = qh.host.slm_config(128)
    blob = qh.host.Blob(cfg, 0xC0F17)
    rng = np.random.default_rng(0xC5)
    prompt = rng.integers(0, cfg.vocab, 64).astype(np.int32)
    got, lg = chunked_device_run(qh, cfg, blob, prompt[None, :], 8)
    want, wl = ref_batch_then_steps(ref, cfg, blob.tensors(), prompt, 8)
    blob.close()
    assert np.array_equal(got[0], want[:8])
    assert np.array_equal(bits(lg[0]), bits(wl[8]))
