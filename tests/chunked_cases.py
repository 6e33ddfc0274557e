# SPDX-License-Identifier: MIT
"""Seeded inputs for the chunked Gated DeltaNet step (slm/chunked.c:287):
per head and token, q and k L2-normalized rows (q also scaled by
1/sqrt(hd)), v of the SiLU'd convolution's range, beta = sigmoid(.) and
g_log = ssm_a * softplus(.) < 0, as slm_forward_ssm_batch forms them
(slm/qwen.c:676-715)."""
import numpy as np


def chunk_inputs(n: int, hd: int, seed: int, state_scale: float = 0.05):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n, hd)).astype(np.float32)
    k = rng.standard_normal((n, hd)).astype(np.float32)
    q = (q / np.linalg.norm(q, axis=1, keepdims=True) / np.sqrt(hd)).astype(np.float32)
    k = (k / np.linalg.norm(k, axis=1, keepdims=True)).astype(np.float32)
    v = rng.standard_normal((n, hd)).astype(np.float32)
    v = (v / (1.0 + np.exp(-v))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal(n)))).astype(np.float32)
    a = rng.standard_normal(n) + 0.5
    g_log = (-np.exp(rng.normal(0.0, 0.02, n)) * np.log1p(np.exp(a))).astype(np.float32)
    state = (rng.standard_normal((hd, hd)) * state_scale).astype(np.float32)
    return q, k, v, g_log, beta, state
