# SPDX-License-Identifier: MIT
"""GPU: the drop-in boundary at work. The reference's unmodified forward
pass (slm_forward_step, compiled from its sources into oracle/_ref) runs
with its matmul entry points (tensor_matmul_q4k/q5k/q6k/q8_0/f32, the
callees of matmul_dispatch, slm/model.c:220-264) replaced by
oracle/libqhdropin.so, which computes them on the GPU through this
library's C-ABI (qh_matmul). Every weight type is exercised (the released
Q4_K_M mix, and a mix with F32 matrices). Bar: the logits of every step are
bit-identical to the stock reference's on the CPU and to the device model's.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("mix,types", [(1, (8, 12, 13, 14)), (2, (0, 8, 13, 14))], ids=["q4_k_m", "all_types"])
def test_reference_forward_with_gpu_matmuls(qh, cuda, ref, tmp_path, mix, types):
    from oracle.oracle import RefModel
    cfg = qh.host.slm_config(32, n_layers=4, vocab=1024)
    blob = qh.host.Blob(cfg, 0xD801 + mix, mix=mix)
    path = str(tmp_path / "m.gguf")
    blob.write_gguf(path)
    prompt, n_new = [5, 77, 300, 2, 999, 41], 8
    out = str(tmp_path / "dropin.npz")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "dropin_child.py"), path,
                        ",".join(map(str, prompt)), str(n_new), out], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.load(out)
    for t in types:
        assert got["calls"][t] > 0, f"no type-{t} matmul went through the GPU"
    # the stock reference on the CPU, same schedule
    rm, _, _ = RefModel.from_gguf(ref, path)
    tok = prompt[0]
    for pos in range(len(prompt) + n_new - 1):
        a, lg = rm.step(tok, pos, want_logits=True)
        assert a == got["preds"][pos]
        assert np.array_equal(lg.view(np.uint32), got["logits"][pos].view(np.uint32)), f"step {pos} logits differ"
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else a
    rm.close()
    # and the device model over the same file
    back = qh.host.Blob.from_gguf(path)
    slm = qh.host.Slm(back.cfg, back, 1)
    tok = np.array([prompt[0]], np.int32)
    for pos in range(len(prompt) + n_new - 1):
        nxt, lg = slm.step(tok, pos, want_logits=True)
        assert np.array_equal(lg[0].view(np.uint32), got["logits"][pos].view(np.uint32)), f"device step {pos}"
        tok = np.array([prompt[pos + 1] if pos + 1 < len(prompt) else nxt[0]], np.int32)
    slm.close()
    back.close()
