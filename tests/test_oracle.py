# SPDX-License-Identifier: MIT
"""CPU: pins the oracle (oracle/qh_oracle.c) to the reference.

1. Against the committed golden fixtures (tests/golden/*.npz, produced by the
   reference's own compiled code via tests/golden/make_golden.py): always
   runs, here and on the GPU box.
2. Against the live reference library oracle/_ref/libqhref.so when it is
   present (skipped otherwise): random blocks, every weight type.
3. Integer per-block sums (isum, isum_mins) checked against a direct
   restatement from the dequantized weights (slm/tensor.c:800-1010).
"""
import glob
import hashlib
import os

import numpy as np
import pytest

from oracle.oracle import Q4_K, Q5_K, Q6_K, Q8_0, to_q8_0_blocks, to_q8k_blocks

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_oracle_matches_golden(path, qh, oracle):
    g = np.load(path)
    gt, k, out_f = int(g["gtype"]), int(g["k"]), int(g["out_f"])
    bw = 32 if gt == Q8_0 else 256
    w = qh.host.synth_blocks(gt, out_f * (k // bw), int(g["wseed"]))
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(g["w_sha256"]), "generator drifted"
    x = g["x"]
    out = oracle.matmul(gt, w, out_f, k, x)
    assert np.array_equal(bits(out), bits(g["out"])), "oracle matmul != reference (bitwise)"
    if gt == Q8_0:
        qs, d = oracle.quantize_q8_0(x)
        assert np.array_equal(qs, g["qs"]) and np.array_equal(d, g["d"])
    else:
        qs, d, bs = oracle.quantize_q8k(x)
        assert np.array_equal(qs, g["qs"]) and np.array_equal(bits(d), bits(g["d"]))
        assert np.array_equal(bs, g["bsums"])
        # reference scalar path == dispatched path for K-quants on x86
        assert np.array_equal(bits(g["scalar_row0"]), bits(g["out"][0]))


def test_golden_edge_cases_present():
    g = np.load([p for p in GOLDEN if "q4k_cfg1" in p][0])
    assert g["d"][0, 1] == 0.0 and not g["qs"][0, 256:512].any(), "all-zero block case missing"
    assert g["qs"][0, 5] == -127 and g["qs"][0, 9] == 127, "signed max / tie case missing"


@pytest.mark.parametrize("gt", [Q4_K, Q5_K, Q6_K, Q8_0])
@pytest.mark.parametrize("k", [256, 1024, 3584])
def test_oracle_vs_live_reference(gt, k, qh, oracle, ref):
    out_f, n_tok = 24, 3
    bw = 32 if gt == Q8_0 else 256
    w = qh.host.synth_blocks(gt, out_f * (k // bw), 77 + k + gt)
    x = qh.host.synth_normal(n_tok * k, 5 + k, 0.0, 3.0).reshape(n_tok, k)
    a = oracle.matmul(gt, w, out_f, k, x)
    b = ref.matmul(gt, w, out_f, k, x)
    assert np.array_equal(bits(a), bits(b))


def test_oracle_q8_0_scalar_order_differs_only_by_ulps(qh, oracle, ref):
    """The AVX tiers' 8-lane order and the scalar order agree to ~ulps."""
    k, out_f = 1024, 32
    w = qh.host.synth_blocks(Q8_0, out_f * k // 32, 4242)
    x = qh.host.synth_normal(k, 17).reshape(1, k)
    qs, d = ref.quantize_q8_0(x)
    blocks = to_q8_0_blocks(qs[0], d[0])
    rb = (k // 32) * 34
    fast = np.array([ref.row_dot(Q8_0, w[j * rb:(j + 1) * rb], blocks, k) for j in range(out_f)])
    slow = np.array([ref.row_dot(Q8_0, w[j * rb:(j + 1) * rb], blocks, k, scalar=True) for j in range(out_f)])
    assert np.allclose(fast, slow, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("gt", [Q4_K, Q5_K, Q6_K])
def test_block_ints_match_dequantized_restatement(gt, qh, oracle):
    """isum / isum_mins against integers rebuilt from the dequant layout rules."""
    rng = np.random.default_rng(3)
    blocks = qh.host.synth_blocks(gt, 8, 900 + gt).reshape(8, -1)
    for blk in blocks:
        q8 = rng.integers(-128, 128, 256, dtype=np.int8)
        bs = q8.reshape(16, 16).astype(np.int32).sum(1).astype(np.int16)
        isum, mins = oracle.block_ints(gt, blk, q8, bs)
        # rebuild integer weights and scales straight from the byte layout
        if gt in (Q4_K, Q5_K):
            s12 = blk[4:16].astype(np.int32)
            sc = np.zeros(8, np.int64)
            mn = np.zeros(8, np.int64)
            for j in range(8):
                if j < 4:
                    sc[j], mn[j] = s12[j] & 63, s12[j + 4] & 63
                else:
                    sc[j] = (s12[j + 4] & 15) | ((s12[j - 4] >> 6) << 4)
                    mn[j] = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4)
            qs = blk[16:144] if gt == Q4_K else blk[48:176]
            w = np.zeros(256, np.int64)
            for c in range(4):
                w[64 * c:64 * c + 32] = qs[32 * c:32 * c + 32] & 15
                w[64 * c + 32:64 * c + 64] = qs[32 * c:32 * c + 32] >> 4
                if gt == Q5_K:
                    qh_ = blk[16:48].astype(np.int64)
                    w[64 * c:64 * c + 32] += ((qh_ >> (2 * c)) & 1) << 4
                    w[64 * c + 32:64 * c + 64] += ((qh_ >> (2 * c + 1)) & 1) << 4
            exp_isum = int(sum(sc[j] * np.dot(w[32 * j:32 * j + 32], q8[32 * j:32 * j + 32].astype(np.int64))
                               for j in range(8)))
            exp_mins = int(sum(mn[j] * (int(bs[2 * j]) + int(bs[2 * j + 1])) for j in range(8)))
        else:
            ql, qhb, sc = blk[0:128].astype(np.int64), blk[128:192].astype(np.int64), blk[192:208].view(np.int8).astype(np.int64)
            w = np.zeros(256, np.int64)
            for h in range(2):
                for l in range(32):
                    a, b_, hb = ql[64 * h + l], ql[64 * h + 32 + l], qhb[32 * h + l]
                    w[128 * h + l] = (a & 15) | ((hb & 3) << 4)
                    w[128 * h + 32 + l] = (b_ & 15) | (((hb >> 2) & 3) << 4)
                    w[128 * h + 64 + l] = (a >> 4) | (((hb >> 4) & 3) << 4)
                    w[128 * h + 96 + l] = (b_ >> 4) | (((hb >> 6) & 3) << 4)
            exp_isum = int(sum(sc[j] * np.dot(w[16 * j:16 * j + 16], q8[16 * j:16 * j + 16].astype(np.int64))
                               for j in range(16)))
            exp_mins = int(np.dot(sc, bs.astype(np.int64)))
        assert (isum, mins) == (exp_isum, exp_mins)


@pytest.mark.parametrize("gt", [Q4_K, Q5_K, Q6_K])
def test_dequant_matches_reference(gt, qh, oracle, ref):
    blocks = qh.host.synth_blocks(gt, 4, 321 + gt).reshape(4, -1)
    for blk in blocks:
        assert np.array_equal(bits(oracle.dequant_block(gt, blk)), bits(ref.dequant_block(gt, blk)))


def test_q8k_blocks_roundtrip_layout(qh, oracle, ref):
    k = 512
    x = qh.host.synth_normal(k, 8)
    qs, d, bs = oracle.quantize_q8k(x.reshape(1, k))
    raw = to_q8k_blocks(qs[0], d[0], bs[0])
    rq = ref.quantize_q8k(x.reshape(1, k))
    assert np.array_equal(raw, to_q8k_blocks(rq[0][0], rq[1][0], rq[2][0]))
