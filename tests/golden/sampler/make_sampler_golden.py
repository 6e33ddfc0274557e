# SPDX-License-Identifier: MIT
"""Generates tests/golden/sampler/sampler.npz from the REFERENCE's own
sampler chain.

    python tests/golden/sampler/make_sampler_golden.py

Runs in the build container, where oracle/_ref/libqhref.so is the
reference compiled from its sources (oracle/Makefile), its expf the host C
library's -- the exponential the device kernel and the oracle evaluate too.
For every case of tests/sampler_cases.py it stores the reference's picks,
generator words and penalized-logits digests (sample_with,
slm/sampler.c:134-180; rng_seed / rng_uniform, slm/model.c:431-447). The
inputs are regenerated from their seeds by the tests.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from conftest import load_pkg  # noqa: E402
from oracle.oracle import Ref  # noqa: E402
import sampler_cases as sc  # noqa: E402


def main():
    host = load_pkg().host
    ref = Ref()
    picks, states, digests, names = [], [], [], []
    for name, vocab, rows in sc.cases():
        p, s, d = sc.run(ref.sample_with, ref.rng_seed, host, name, vocab, rows)
        picks.append(p)
        states.append(s)
        digests.extend(d)
        names.append(f"{name}/{vocab}")
    out = os.path.join(HERE, "sampler.npz")
    np.savez_compressed(out, picks=np.stack(picks), states=np.stack(states), digests=np.array(digests),
                        names=np.array(names))
    print("wrote", out, np.stack(picks).shape)


if __name__ == "__main__":
    main()
