# SPDX-License-Identifier: MIT
"""Generates tests/golden/*.npz from the REFERENCE's own C code.

    python tests/golden/make_golden.py

Runs in the build container, where oracle/_ref/libqhref.so is compiled from
the qwen.haiku sources (oracle/Makefile). Each fixture holds the inputs that
cannot be regenerated bit-for-bit elsewhere (activations) plus the
reference's outputs; weight bytes are regenerated from their seed with the
integer-only generator of include/qh_synth.h and checked against the stored
SHA-256. Reference entry points used:
  ref_matmul        -> matmul_dispatch / tensor_matmul_*_f32 (slm/model.c:220,
                       slm/tensor.c:827-1033), dispatched SIMD tier
  ref_row_dot(scalar) -> q_scalar_*_dot (simd/quants.h:244-402)
  ref_quantize_*    -> quantize_row_q8_K / tensor_quantize_row_q8_0
                       (slm/tensor.c:683, 930)
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from conftest import load_pkg  # noqa: E402
from oracle.oracle import Ref, to_q8_0_blocks, to_q8k_blocks  # noqa: E402

Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14

# (name, type, k, out_f, n_tok, weight seed, activation seed)
CASES = [
    ("q4k_cfg1", Q4_K, 1024, 3072, 1, 0x5EED01, 0xA0),
    ("q4k_small", Q4_K, 256, 40, 3, 0x5EED11, 0xA1),
    ("q5k_attn_out", Q5_K, 2048, 256, 2, 0x5EED21, 0xA2),
    ("q6k_down", Q6_K, 3584, 128, 2, 0x5EED31, 0xA3),
    ("q6k_k1024", Q6_K, 1024, 72, 1, 0x5EED32, 0xA4),
    ("q8_0_sq", Q8_0, 1024, 96, 2, 0x5EED41, 0xA5),
    ("q8_0_k32", Q8_0, 32, 24, 1, 0x5EED42, 0xA6),
]


def edge_activations(k: int, n_tok: int, seed: int, host) -> np.ndarray:
    """N(0,1)-shaped rows plus the quantizer's edge cases in row 0."""
    x = host.synth_normal(n_tok * k, seed).reshape(n_tok, k)
    r0 = x[0]
    if k >= 512:
        r0[256:512] = 0.0                    # all-zero Q8_K block -> d = 0
    r0[5] = -7.25                            # signed max-magnitude
    r0[9] = 7.25                             # tie in magnitude: first index wins
    r0[17] = 0.5 * 7.25 / 127.0 * 3.0        # lands near a .5 rounding boundary
    return x.astype(np.float32)


def main() -> None:
    qh = load_pkg()
    host = qh.host
    ref = Ref()
    for name, gt, k, out_f, n_tok, wseed, xseed in CASES:
        bw = 32 if gt == Q8_0 else 256
        w = host.synth_blocks(gt, out_f * (k // bw), wseed)
        x = edge_activations(k, n_tok, xseed, host)
        out = ref.matmul(gt, w, out_f, k, x)
        if gt == Q8_0:
            qs, d = ref.quantize_q8_0(x)
            bs = np.zeros((n_tok, 0), np.int16)
            xq0 = to_q8_0_blocks(qs[0], d[0])
        else:
            qs, d, bs = ref.quantize_q8k(x)
            xq0 = to_q8k_blocks(qs[0], d[0], bs[0])
        rb = (k // bw) * {Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_0: 34}[gt]
        scalar0 = np.array([ref.row_dot(gt, w[j * rb:(j + 1) * rb], xq0, k, scalar=True)
                            for j in range(out_f)], np.float32)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            gtype=gt, k=k, out_f=out_f, n_tok=n_tok, wseed=wseed,
            w_sha256=hashlib.sha256(w.tobytes()).hexdigest(),
            x=x, out=out, qs=qs, d=d, bsums=bs, scalar_row0=scalar0,
            dispatch=ref.label)
        print(f"{name}: type {gt} k {k} out_f {out_f} n_tok {n_tok} dispatch {ref.label}")


if __name__ == "__main__":
    main()
