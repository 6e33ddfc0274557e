# SPDX-License-Identifier: MIT
"""Child process of tests/test_dropin_gpu.py: the reference's own forward
pass (slm_forward_step, oracle/_ref/libqhref.so) with its tensor_matmul_*
entry points replaced by oracle/libqhdropin.so, which computes them on the
GPU through libqh200.so's C-ABI. Runs in a fresh process because the
replacement is process-wide (the shim is loaded with RTLD_GLOBAL before the
reference library).

    python tests/dropin_child.py MODEL.gguf PROMPT_IDS(comma) N_NEW OUT.npz
"""
import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    path, prompt, n_new, out = sys.argv[1], [int(t) for t in sys.argv[2].split(",")], int(sys.argv[3]), sys.argv[4]
    shim = C.CDLL(os.path.join(ROOT, "oracle", "libqhdropin.so"), mode=C.RTLD_GLOBAL)
    shim.dropin_init.argtypes = [C.c_char_p, C.c_char_p]
    shim.dropin_calls.restype = C.c_int64
    from oracle.oracle import REF_SO, Ref, RefModel
    ref = Ref()
    qh = os.path.join(ROOT, "qwen.haiku_b200", "libqh200.so")
    assert shim.dropin_init(REF_SO.encode(), qh.encode()) == 0, "dropin_init failed"
    rm, _, _ = RefModel.from_gguf(ref, path)
    preds, logits = [], []
    tok = prompt[0]
    for pos in range(len(prompt) + n_new - 1):
        a, lg = rm.step(tok, pos, want_logits=True)
        preds.append(a)
        logits.append(lg.copy())
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else a
    rm.close()
    calls = np.array([shim.dropin_calls(t) for t in range(16)], np.int64)
    np.savez(out, preds=np.array(preds, np.int32), logits=np.stack(logits), calls=calls)


if __name__ == "__main__":
    main()
