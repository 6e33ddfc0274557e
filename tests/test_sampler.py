# SPDX-License-Identifier: MIT
"""The sampler chain (include/qh_sampler.h) against the reference's
sample_with (slm/sampler.c:134-180).

CPU: the restatement in oracle/qh_oracle.c against the committed golden
picks (tests/golden/sampler/sampler.npz, made by the reference compiled from its
sources, expf the host C library's) and against the live reference; the
product's host-side helpers (defaults, generator seeding).
GPU: qh_sample on the device against the same golden picks, generator words
and penalized logits, three successive draws per row with the generator
carried over, for every case of tests/sampler_cases.py.
Bar: bit-exact (picks, generator words and penalized logits bytes).
"""
import hashlib
import os

import numpy as np
import pytest

import sampler_cases as sc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampler", "sampler.npz")
CASES = sc.cases()


def golden():
    return np.load(GOLDEN)


def test_defaults_match_reference(qh, ref):
    got = qh.host.sampler_defaults().as_dict()
    want = ref.sampler_defaults()
    for f, v in want.items():
        assert np.float32(got[f]) == np.float32(v), f


@pytest.mark.parametrize("seed", [0, 1, 0x5EED, 2**63 + 5, 2**64 - 1, 0x9E3779B97F4A7C15 * 3 % 2**64])
def test_rng_seed_matches_reference(qh, ref, seed):
    assert np.array_equal(qh.host.rng_seed(seed), ref.rng_seed(seed))


@pytest.mark.parametrize("ci", range(len(CASES)), ids=[f"{c[0]}-{c[1]}" for c in CASES])
def test_oracle_sampler_matches_golden(qh, oracle, ci):
    name, vocab, rows = CASES[ci]
    g = golden()
    assert str(g["names"][ci]) == f"{name}/{vocab}"
    picks, states, digests = sc.run(oracle.sample_with, qh.host.rng_seed, qh.host, name, vocab, rows)
    assert np.array_equal(picks, g["picks"][ci])
    assert np.array_equal(states, g["states"][ci])
    n = len(rows) * sc.CALLS
    assert digests == [str(d) for d in g["digests"][ci * n:(ci + 1) * n]]


@pytest.mark.parametrize("ci", [0, 5, 9, 14])
def test_oracle_sampler_matches_live_reference(qh, oracle, ref, ci):
    name, vocab, rows = CASES[ci]
    a = sc.run(oracle.sample_with, qh.host.rng_seed, qh.host, name, vocab, rows)
    b = sc.run(ref.sample_with, ref.rng_seed, qh.host, name, vocab, rows)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and a[2] == b[2]


def test_golden_covers_edge_cases():
    g = golden()
    names = [str(n) for n in g["names"]]
    for want in ("defaults/151936", "k_over_max/100", "greedy_pen/4096", "k1/151936"):
        assert want in names
    kinds = {r[0] for c in CASES for r in c[2]}
    assert kinds == set(sc.KINDS)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def device_run(qh, torch, name, vocab, rows):
    """sc.run's schedule on the device: all rows in one qh_sample launch per
    call; the history and generator live in device memory."""
    sp = qh.Sampler(**sc.SAMPLERS[name])
    B = len(rows)
    stride = max(r[2] for r in rows) + sc.CALLS + 1
    hist = np.zeros((B, stride), np.int32)
    hn = np.zeros(B, np.int32)
    for b, (_, _, hlen, hseed) in enumerate(rows):
        hist[b, :hlen] = sc.history(vocab, hlen, hseed)
        hn[b] = hlen
    st = np.stack([qh.host.rng_seed(s) for s in sc.RNG_SEEDS[:B]]).view(np.int64)
    d_hist, d_hn = torch.from_numpy(hist).cuda(), torch.from_numpy(hn).cuda()
    d_rng = torch.from_numpy(st.copy()).cuda()
    picks = np.zeros((B, sc.CALLS), np.int32)
    states = np.zeros((B, sc.CALLS, 2), np.uint64)
    digests = [[None] * sc.CALLS for _ in range(B)]
    for call in range(sc.CALLS):
        lg = np.stack([sc.logits(qh.host, kind, vocab, lseed + 7919 * call) for kind, lseed, _, _ in rows])
        d_lg = torch.from_numpy(lg).cuda()
        out = qh.host.sample(sp, d_lg, d_hist, d_hn, d_rng)
        torch.cuda.synchronize()
        p = out.cpu().numpy()
        picks[:, call] = p
        states[:, call] = d_rng.cpu().numpy().view(np.uint64)
        pen = d_lg.cpu().numpy()
        for b in range(B):
            digests[b][call] = hashlib.sha256(np.ascontiguousarray(pen[b]).tobytes()).hexdigest()
            hist[b, hn[b]] = p[b]
            hn[b] += 1
        d_hist.copy_(torch.from_numpy(hist))
        d_hn.copy_(torch.from_numpy(hn))
    qh.check(qh.lib().qh_check_device_error(None), "device error word")
    return picks, states, [d for row in digests for d in row]


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(len(CASES)), ids=[f"{c[0]}-{c[1]}" for c in CASES])
def test_device_sampler_matches_reference(qh, cuda, ci):
    name, vocab, rows = CASES[ci]
    g = golden()
    picks, states, digests = device_run(qh, cuda, name, vocab, rows)
    assert np.array_equal(picks, g["picks"][ci]), f"picks {picks.tolist()} != {g['picks'][ci].tolist()}"
    assert np.array_equal(states, g["states"][ci])
    n = len(rows) * sc.CALLS
    assert digests == [str(d) for d in g["digests"][ci * n:(ci + 1) * n]], "penalized logits differ"


@pytest.mark.gpu
def test_device_sampler_many_rows(qh, cuda, oracle):
    """64 rows in one launch (one CTA each), default settings, full vocabulary."""
    torch = cuda
    B, vocab = 64, 151936
    sp = qh.host.sampler_defaults()
    lg = np.stack([sc.logits(qh.host, sc.KINDS[b % len(sc.KINDS)], vocab, 9000 + b) for b in range(B)])
    hist = np.stack([sc.history(vocab, 70, 400 + b) for b in range(B)])
    hn = np.full(B, 70, np.int32)
    st = np.stack([qh.host.rng_seed(b + 1) for b in range(B)])
    d_lg = torch.from_numpy(lg.copy()).cuda()
    d_rng = torch.from_numpy(st.view(np.int64).copy()).cuda()
    out = qh.host.sample(sp, d_lg, torch.from_numpy(hist).cuda(), torch.from_numpy(hn).cuda(), d_rng)
    got = out.cpu().numpy()
    spd = sp.as_dict()
    for b in range(B):
        s = st[b].copy()
        want = oracle.sample_with(np.ascontiguousarray(lg[b]), spd, s, hist[b])
        assert got[b] == want, f"row {b}"
        assert np.array_equal(d_rng[b].cpu().numpy().view(np.uint64), s)


def ref_generate(ref, RefModel, cfg, tensors, prompt, max_new, min_new, sp, seed, eos, eot, stops):
    """slm_generate_raw (slm/slm.c:237-357) with the reference's own
    slm_forward_step and sample_with: prompt at positions 0..n-1, then the
    decode loop re-feeding the last prompt token at position n."""
    rm = RefModel(ref, cfg, tensors)
    for i, t in enumerate(prompt):
        rm.step(int(t), i)
    st = ref.rng_seed(seed)
    hist, out, pos, last = [int(t) for t in prompt], [], len(prompt), int(prompt[-1])
    while len(out) < max_new and pos < cfg.max_pos:
        _, lg = rm.step(last, pos, want_logits=True)
        if len(out) < min_new:
            for t in (eos, eot):
                if 0 <= t < cfg.vocab:
                    lg[t] = -np.inf
        nxt = ref.sample_with(lg, sp, st, np.array(hist, np.int32))
        hist.append(nxt)
        out.append(nxt)
        pos += 1
        if nxt in (eos, eot) or nxt in stops:
            break
        last = nxt
    rm.close()
    return np.array(out, np.int32)


@pytest.mark.gpu
@pytest.mark.parametrize("setting", ["defaults", "k256_plain", "tight"])
def test_generate_sampled_matches_reference(qh, cuda, ref, setting):
    """qh_slm_generate_sampled on three sequences against the reference's
    generation loop, token for token (small 4-layer model, vocab 4096).
    eos/eot are set to tokens the model favours, so the min_new masking and
    the stop rule both take effect."""
    from oracle.oracle import RefModel
    cfg = qh.host.slm_config(48, n_layers=4, vocab=4096)
    blob = qh.host.Blob(cfg, 0x5A3B1)
    tensors = blob.tensors()
    rng = np.random.default_rng(11)
    B, n_prompt, max_new, min_new = 3, 9, 30, 4
    prompts = rng.integers(0, cfg.vocab, (B, n_prompt)).astype(np.int32)
    seeds = np.array([7, 0x5EED, 2**40 + 3], np.uint64)
    sp = qh.Sampler(**sc.SAMPLERS[setting])
    # eos/eot: the first two tokens the unconstrained sampler emits for sequence 0
    slm = qh.host.Slm(cfg, blob, B)
    free = slm.generate_sampled(prompts, 6, sp, seeds)
    eos, eot = int(free[0][1]), int(free[0][3])
    stops = (int(free[1][5]),)
    got = slm.generate_sampled(prompts, max_new, sp, seeds, min_new=min_new, eos_id=eos, eot_id=eot,
                               stop_ids=stops)
    again = slm.generate_sampled(prompts, max_new, sp, seeds, min_new=min_new, eos_id=eos, eot_id=eot,
                                 stop_ids=stops)
    slm.close()
    for b in range(B):
        want = ref_generate(ref, RefModel, cfg, tensors, prompts[b], max_new, min_new, sp.as_dict(),
                            int(seeds[b]), eos, eot, stops)
        assert np.array_equal(got[b], want), f"sequence {b}: {got[b].tolist()} != {want.tolist()}"
        assert np.array_equal(again[b], got[b]), "re-seeded run differs"


@pytest.mark.gpu
def test_generate_sampled_continues_generator(qh, cuda):
    """seeds = 0 continues each sequence's generator: two calls without a
    seed differ, and re-seeding reproduces the first."""
    cfg = qh.host.slm_config(48, n_layers=4, vocab=4096)
    blob = qh.host.Blob(cfg, 0x5A3B1)
    slm = qh.host.Slm(cfg, blob, 2)
    prompts = np.arange(10, dtype=np.int32).reshape(2, 5) * 37
    sp = qh.Sampler(**sc.SAMPLERS["k256_plain"])
    first = slm.generate_sampled(prompts, 12, sp, np.array([99, 98], np.uint64))
    cont = slm.generate_sampled(prompts, 12, sp, None)
    again = slm.generate_sampled(prompts, 12, sp, np.array([99, 98], np.uint64))
    slm.close()
    assert any(not np.array_equal(a, b) for a, b in zip(first, cont))
    assert all(np.array_equal(a, b) for a, b in zip(first, again))
