# SPDX-License-Identifier: MIT
"""Generates tests/golden/chunked/chunked.npz from the REFERENCE's own
chunked Gated DeltaNet step (chunked_ssm_step_f32, slm/chunked.c:287-523,
compiled from its sources into oracle/_ref by oracle/Makefile), run in
slm_forward_ssm_batch's 64-token chunk loop from a zero state.

    python tests/golden/chunked/make_chunked_golden.py

Stores the inputs, the outputs and the SHA-256 of the final state's bytes
(expf from the host C library, as the reference is built).
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, ROOT)

from oracle.oracle import Ref  # noqa: E402
from tests.chunked_cases import chunk_inputs  # noqa: E402

# (name, tokens, head dim, seed): two chunks (the second ragged) and one short chunk
CASES = [("c70_hd64", 70, 64, 0xC401), ("c9_hd128", 9, 128, 0xC402)]


def main():
    ref = Ref()
    out = {}
    for name, n, hd, seed in CASES:
        q, k, v, g, b, _ = chunk_inputs(n, hd, seed)
        for key, a in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", b)):
            out[f"{name}_{key}"] = a
        st = np.zeros((hd, hd), np.float32)
        out[f"{name}_out"] = ref.chunked_prefill(q, k, v, g, b, st)
        out[f"{name}_state_sha"] = np.array(hashlib.sha256(st.tobytes()).hexdigest())
    np.savez_compressed(os.path.join(HERE, "chunked.npz"), **out)
    print("wrote", os.path.join(HERE, "chunked.npz"))


if __name__ == "__main__":
    main()
