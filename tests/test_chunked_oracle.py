# SPDX-License-Identifier: MIT
"""CPU: pins the oracle's chunked Gated DeltaNet step (orc_chunked_step in
oracle/qh_oracle.c) to the reference's own chunked_ssm_step_f32
(slm/chunked.c:287-523, compiled from its sources into oracle/_ref), run in
slm_forward_ssm_batch's 64-token chunk loop with the state carried
(slm/qwen.c:777-806). Bit-exact, outputs and final state, both on the
host C library's expf."""
import os

import numpy as np
import pytest

from tests.chunked_cases import chunk_inputs


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("n", [1, 2, 17, 63, 64, 65, 130, 200])
def test_oracle_chunked_matches_reference(n, oracle, ref):
    q, k, v, g, b, s0 = chunk_inputs(n, 128, 1000 + n)
    s_ref, s_orc = s0.copy(), s0.copy()
    o_ref = ref.chunked_prefill(q, k, v, g, b, s_ref)
    o_orc = oracle.chunked_prefill(q, k, v, g, b, s_orc)
    assert np.array_equal(bits(o_orc), bits(o_ref)), "chunk outputs differ from the reference"
    assert np.array_equal(bits(s_orc), bits(s_ref)), "carried state differs from the reference"


def test_oracle_chunked_small_head_and_zero_state(oracle, ref):
    q, k, v, g, b, _ = chunk_inputs(70, 32, 7)
    s_ref = np.zeros((32, 32), np.float32)
    s_orc = s_ref.copy()
    o_ref = ref.chunked_prefill(q, k, v, g, b, s_ref)
    o_orc = oracle.chunked_prefill(q, k, v, g, b, s_orc)
    assert np.array_equal(bits(o_orc), bits(o_ref)) and np.array_equal(bits(s_orc), bits(s_ref))


def test_chunked_close_to_recurrent_update(oracle):
    """The chunked algebra is the delta rule: against a float64 token-by-token
    recurrence S <- g S + k (beta (v - S^T k g))^T, out = S^T q, it agrees to
    float rounding (the reference's chunked-test bar is 1e-5 relative)."""
    n, hd = 130, 128
    q, k, v, g, b, s0 = chunk_inputs(n, hd, 3)
    s = s0.copy()
    out = oracle.chunked_prefill(q, k, v, g, b, s)
    S = s0.astype(np.float64)
    want = np.empty((n, hd))
    for t in range(n):
        S *= np.exp(np.float64(g[t]))
        delta = b[t] * (v[t] - S.T @ k[t])
        S += np.outer(k[t], delta)
        want[t] = S.T @ q[t]
    rel = np.abs(out - want).max() / np.abs(want).max()
    assert rel < 1e-5, f"chunked vs recurrent relative difference {rel:.2e}"
    assert np.abs(s - S).max() / np.abs(S).max() < 1e-5


@pytest.mark.parametrize("n", [0, 65])
def test_chunk_step_rejects_sizes_outside_one_chunk(n, oracle, ref):
    """Both the reference wrapper and the oracle take 1..64 tokens per call
    (CHUNK_SIZE, slm/chunked.c:116); larger prompts go through the chunk loop."""
    import ctypes as C
    hd = 128
    a = np.zeros((max(n, 1), hd), np.float32)
    v = np.zeros(max(n, 1), np.float32)
    s = np.zeros((hd, hd), np.float32)
    o = np.zeros((max(n, 1), hd), np.float32)
    P = lambda x: C.c_void_p(x.ctypes.data)
    assert oracle.L.orc_chunked_step(n, hd, P(a), P(a), P(a), P(v), P(v), P(s), P(o)) == -1
    assert ref.L.ref_chunked_step(n, hd, hd, P(a), P(a), P(a), P(v), P(v), P(s), P(o)) == -1


GOLDEN_CHUNKED = os.path.join(os.path.dirname(__file__), "golden", "chunked", "chunked.npz")


@pytest.mark.parametrize("name", ["c70_hd64", "c9_hd128"])
def test_oracle_chunked_matches_golden(name, oracle):
    """Against fixtures the reference's own chunk step wrote
    (tests/golden/chunked/make_chunked_golden.py): runs without the
    reference library, here and on the GPU box."""
    import hashlib
    g = np.load(GOLDEN_CHUNKED)
    q, k, v, gl, b = (g[f"{name}_{x}"] for x in ("q", "k", "v", "g", "beta"))
    hd = q.shape[1]
    st = np.zeros((hd, hd), np.float32)
    out = oracle.chunked_prefill(q, k, v, gl, b, st)
    assert np.array_equal(bits(out), bits(g[f"{name}_out"])), "outputs differ from the reference's"
    assert hashlib.sha256(st.tobytes()).hexdigest() == str(g[f"{name}_state_sha"]), "final state differs"
