# SPDX-License-Identifier: MIT
"""CPU: the C-ABI library loads, exports every symbol include/*.h declares,
and host-only entry points behave (no GPU compute here)."""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b(qh_\w+|slm_\w+)\s*\(", text):
            # keep declarations (a return type before the name), not macro uses
            start = text.rfind("\n", 0, m.start()) + 1
            prefix = text[start:m.start()].strip()
            if prefix and not prefix.startswith("#") and not prefix.endswith(("=", ",", "(")):
                names.add(m.group(1))
    return sorted(names)


def test_headers_found():
    assert any(h.endswith("qh_backend.h") for h in HEADERS)
    assert len(declared_functions()) >= 30


@pytest.mark.parametrize("name", declared_functions())
def test_symbol_exported(qh, name):
    L = qh.lib()
    assert hasattr(L, name), f"{name} declared in include/ but not exported by libqh200.so"


def test_bindings_cover_every_declaration(qh):
    missing = [n for n in declared_functions() if n not in qh.SIGNATURES]
    assert not missing, f"ctypes signatures missing for {missing}"


def test_version_and_device_count(qh):
    assert b"sm_100a" in qh.lib().qh_version()
    assert qh.lib().qh_device_count() >= 0


def test_layout_sizes(qh):
    L = qh.lib()
    # Q8_K split: qs k*n, d (k/256)*n f32, bsums (k/16)*n int16, 16-byte aligned planes
    k, n = 1024, 3
    assert L.qh_q8k_d_offset(k, n) == 3072
    assert L.qh_q8k_bsums_offset(k, n) == 3072 + 48
    assert L.qh_q8k_bytes(k, n) == 3072 + 48 + 384
    assert L.qh_q8_0_d_offset(k, n) == 3072
    assert L.qh_q8_0_bytes(k, n) == 3072 + 192
    assert L.qh_matmul_workspace_bytes(qh.Q4_K, k, n) == L.qh_q8k_bytes(k, n)
    assert L.qh_matmul_workspace_bytes(qh.Q8_0, k, n) == L.qh_q8_0_bytes(k, n)
    assert L.qh_matmul_workspace_bytes(99, k, n) == -1


def test_argument_errors_before_device(qh):
    """Shape/type errors are reported without touching a device."""
    L = qh.lib()
    p = C.c_void_p(16)
    rc = L.qh_matmul(99, p, 1024, 8, p, 1, p, p, 1 << 20, None)
    assert rc == -2 and b"unsupported" in L.qh_last_error()
    rc = L.qh_matmul(qh.Q4_K, p, 1000, 8, p, 1, p, p, 1 << 20, None)
    assert rc == -1
    rc = L.qh_matmul(qh.Q4_K, C.c_void_p(0), 1024, 8, p, 1, p, p, 1 << 20, None)
    assert rc == -1
    rc = L.qh_matmul(qh.Q4_K, C.c_void_p(18), 1024, 8, p, 1, p, p, 1 << 20, None)
    assert rc == -4
    rc = L.qh_matmul(qh.Q4_K, p, 1024, 8, p, 1, p, p, 16, None)
    assert rc == -5
    rc = L.qh_matvec_plan_create(qh.Q4_K, None, 0, 1, C.byref(C.c_void_p()))
    assert rc == -1


def test_synth_deterministic(qh):
    h = qh.host
    a = h.synth_blocks(qh.Q4_K, 16, 7)
    b = h.synth_blocks(qh.Q4_K, 16, 7)
    assert np.array_equal(a, b) and not np.array_equal(a, h.synth_blocks(qh.Q4_K, 16, 8))
    assert qh.lib().qh_synth_u64(1, 0) == qh.lib().qh_synth_u64(1, 0)
    x = h.synth_normal(200000, 3)
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01
    assert float(np.abs(x).max()) <= 6.0
    # fp16 scale fields land in [1e-3, 1e-2]
    blk = a.reshape(16, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float32)
    assert (d >= 0.000999).all() and (d <= 0.01001).all()


@pytest.mark.parametrize("gt", [12, 13, 14, 8])
def test_synth_quantizer_roundtrip(qh, oracle, gt):
    """The synthetic-model quantizer emits blocks whose dequantization tracks
    the fp32 weights (quality is not a parity requirement, sanity only)."""
    w = qh.host.synth_normal(4 * 256, 11, 0.0, 0.02).reshape(4, 256)
    blocks = qh.host.synth_quantize(gt, w)
    if gt == 8:
        raw = blocks.reshape(4 * 8, 34)
        d = raw[:, 0:2].copy().view(np.float16).astype(np.float32)
        deq = (raw[:, 2:].view(np.int8).astype(np.float32) * d).reshape(4, 256)
    else:
        bb = {12: 144, 13: 176, 14: 210}[gt]
        deq = np.stack([oracle.dequant_block(gt, blocks[i * bb:(i + 1) * bb]) for i in range(4)])
    err = np.abs(deq - w).max() / np.abs(w).max()
    assert err < {12: 0.12, 13: 0.06, 14: 0.04, 8: 0.01}[gt], err


def test_chunked_prefill_entry_points_reject_bad_arguments_on_host(qh):
    """The chunked DeltaNet launchers and the prefill-mode switch check their
    arguments before any device work (status codes, no abort)."""
    L = qh.lib()
    INVALID, UNSUPPORTED = -1, -2
    fake = C.c_void_p(0x1000)  # never dereferenced: the checks fail first
    assert L.qh_gdn_chunked(None, None, None, None, 1, 1, 1, 128, None, None) == INVALID
    assert L.qh_gdn_chunked(fake, fake, fake, fake, 1, 0, 1, 128, fake, None) == INVALID  # no tokens
    assert L.qh_gdn_chunked(fake, fake, fake, fake, 1, 1, 1, 64, fake, None) == UNSUPPORTED  # head dim
    assert L.qh_gdn_chunk_prep(None, None, None, None, None, None, None, 1, 1, 1, 128, 4, None, None) == INVALID
    assert L.qh_gdn_chunk_prep(fake, fake, fake, fake, fake, fake, fake, 1, 1, 1, 128, 3, fake, None) == UNSUPPORTED
    assert L.qh_slm_set_prefill_mode(None, qh.PREFILL_CHUNKED) == INVALID
    assert L.qh_matvec_plan_fuse_output(None, 1, 1024, None, None, None, 0.0, None, None) == INVALID


def test_bad_device_id_is_a_status(qh):
    """A device id the machine does not have is reported, not aborted on."""
    L = qh.lib()
    assert L.qh_set_device(4096) != 0
    assert len(L.qh_last_error()) > 0
