# SPDX-License-Identifier: MIT
"""Seeded inputs for the sampler-chain parity tests (sample_with,
slm/sampler.c:134-180): logits rows, token histories and sampler settings.

Logits come from the repository's own seeded generator (host.synth_normal),
so every machine regenerates the same bytes; the histories use a tiny
integer generator of their own. Shared by tests/test_sampler.py and
tests/golden/make_sampler_golden.py.
"""
from __future__ import annotations

import numpy as np

# name -> sampler settings (struct slm_sampler fields)
SAMPLERS = {
    "defaults": dict(temperature=0.7, top_k=40, top_p=0.9, min_p=0.05, repetition_penalty=1.25,
                     repetition_window=64),
    "k256_plain": dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, repetition_penalty=1.0,
                       repetition_window=0),
    "k_over_max": dict(temperature=1.5, top_k=300, top_p=0.95, min_p=0.0, repetition_penalty=1.1,
                       repetition_window=0),
    "k1": dict(temperature=0.9, top_k=1, top_p=0.9, min_p=0.05, repetition_penalty=1.25, repetition_window=8),
    "greedy_pen": dict(temperature=0.0, top_k=40, top_p=0.9, min_p=0.05, repetition_penalty=1.3,
                       repetition_window=16),
    "tight": dict(temperature=0.3, top_k=256, top_p=0.5, min_p=0.2, repetition_penalty=0.8,
                  repetition_window=200),
}

VOCABS = (151936, 4096, 100)
KINDS = ("normal", "ties", "neg_inf", "peaked", "flat")


def _lcg(seed: int, n: int, mod: int) -> np.ndarray:
    """n integers in [0, mod) from a 64-bit LCG (Knuth's MMIX constants)."""
    out = np.empty(n, np.int64)
    x = (seed * 2654435761 + 1) & ((1 << 64) - 1)
    for i in range(n):
        x = (x * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        out[i] = (x >> 33) % mod
    return out


def logits(host, kind: str, vocab: int, seed: int) -> np.ndarray:
    """One float32 logits row of the given kind."""
    x = host.synth_normal(vocab, seed, 0.0, 3.0).astype(np.float32)
    if kind == "ties":  # quarter steps: many equal values, ties inside the top-k
        x = (np.round(x * 4.0) / 4.0).astype(np.float32)
    elif kind == "neg_inf":  # masked entries, e.g. an eos held back
        idx = _lcg(seed + 1, max(1, vocab // 10), vocab)
        x[idx] = -np.inf
    elif kind == "peaked":  # one dominant token
        x[int(_lcg(seed + 2, 1, vocab)[0])] += 40.0
    elif kind == "flat":  # every logit equal (+0 and -0 mixed): first-slot ties everywhere
        x[:] = 0.0
        x[_lcg(seed + 3, max(1, vocab // 3), vocab)] = -0.0
    return np.ascontiguousarray(x)


def history(vocab: int, n: int, seed: int) -> np.ndarray:
    """n token ids drawn from a small pool (so tokens repeat), with a few
    out-of-range ids the reference skips."""
    if n == 0:
        return np.zeros(0, np.int32)
    pool = _lcg(seed, 24, vocab)
    h = pool[_lcg(seed + 5, n, 24)]
    if n > 4:
        h[1] = -1
        h[n // 2] = vocab + 3
    return h.astype(np.int32)


HIST_LENS = (0, 5, 100, 300)


def cases():
    """(sampler name, vocab, [(kind, logits seed, history length, history seed)] rows)."""
    out = []
    for si, name in enumerate(SAMPLERS):
        for vi, vocab in enumerate(VOCABS):
            rows = []
            for r in range(3):
                kind = KINDS[(si + vi + r) % len(KINDS)]
                rows.append((kind, 1000 * si + 100 * vi + r, HIST_LENS[(si + r) % len(HIST_LENS)], 77 + 10 * si + r))
            out.append((name, vocab, rows))
    return out


CALLS = 3            # successive draws per row, the generator carried over
RNG_SEEDS = (0x5EED, 1, 0xFFFFFFFFFFFFFFFF)  # one per row


def run(sampler_fn, rng_seed_fn, host, name: str, vocab: int, rows):
    """Plays every row of a case through `sampler_fn(logits, sp, st, hist)`
    (the reference's sample_with or a restatement): CALLS successive draws
    per row with fresh logits, each pick appended to the history. Returns
    picks [rows][CALLS], generator words [rows][CALLS][2] after each draw and
    the SHA-256 of each penalized logits row."""
    import hashlib
    sp = SAMPLERS[name]
    picks = np.zeros((len(rows), CALLS), np.int32)
    states = np.zeros((len(rows), CALLS, 2), np.uint64)
    digests = []
    for r, (kind, lseed, hlen, hseed) in enumerate(rows):
        st = rng_seed_fn(RNG_SEEDS[r])
        h = list(history(vocab, hlen, hseed))
        for call in range(CALLS):
            lg = logits(host, kind, vocab, lseed + 7919 * call)
            p = sampler_fn(lg, sp, st, np.array(h, np.int32))
            picks[r, call] = p
            states[r, call] = st
            digests.append(hashlib.sha256(lg.tobytes()).hexdigest())
            h.append(p)
    return picks, states, digests
