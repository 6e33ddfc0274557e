# SPDX-License-Identifier: MIT
"""GPU: qh_matmul_q4k_f32_noalloc, the Q4_K matmul for callers that may not
allocate device memory (a host that owns all device memory in its own pool,
or one that forbids cudaMalloc after start-up because an allocation can
synchronize the device). It keeps its activation scratch in a fixed device
array inside the library instead of a caller workspace.

Checked through the C-ABI on two calls in a row -- the second call reuses the
array the first one left behind -- against the CPU oracle (the reference's
quantizer and row dots restated) with the suite's bar for this path:
bit-identical fp32 outputs; and against the regular workspace entry point
(qh_matmul_q4k_f32). After the calls the library's error check reads the
array's error word and must report no kernel error. This file is named to be
collected last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q4_K = 12


def _call_both(qh, torch, w, x, k, out_f, n_tok):
    L = qh.lib()
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    out_ref = torch.empty((n_tok, out_f), dtype=torch.float32, device="cuda")
    out_new = torch.full((n_tok, out_f), float("nan"), dtype=torch.float32, device="cuda")
    need = int(L.qh_matmul_workspace_bytes(Q4_K, k, n_tok))
    work = torch.empty(need, dtype=torch.uint8, device="cuda")
    qh.check(L.qh_matmul_q4k_f32(C.c_void_p(w.data_ptr()), out_f, k, C.c_void_p(x.data_ptr()), n_tok,
                                 C.c_void_p(out_ref.data_ptr()), C.c_void_p(work.data_ptr()), need, s),
             "qh_matmul_q4k_f32")
    qh.check(L.qh_matmul_q4k_f32_noalloc(C.c_void_p(w.data_ptr()), out_f, k, C.c_void_p(x.data_ptr()),
                                         n_tok, C.c_void_p(out_new.data_ptr()), s),
             "qh_matmul_q4k_f32_noalloc")
    torch.cuda.synchronize()
    return out_ref.cpu().numpy(), out_new.cpu().numpy()


# (8192, 8): a stage cannot hold 8 rows of k = 8192, so the launches take
# fewer tokens each -- the chunking of the workspace entry point.
@pytest.mark.parametrize("k,out_f,n_tok", [(1024, 3072, 1), (3584, 200, 3), (256, 40, 11), (8192, 64, 8)])
def test_noalloc_matches_oracle_two_calls(qh, cuda, oracle, k, out_f, n_tok):
    torch = cuda
    h = qh.host
    for call in range(2):
        w_np = h.synth_blocks(Q4_K, out_f * (k // 256), 0xA110C + 17 * call + k)
        x_np = h.synth_normal(n_tok * k, 0xB0B + 31 * call + n_tok).reshape(n_tok, k)
        want = np.asarray(oracle.matmul(Q4_K, w_np, out_f, k, x_np), np.float32).reshape(n_tok, out_f)
        ws, got = _call_both(qh, torch, h.to_device(w_np), h.to_device(x_np), k, out_f, n_tok)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"call {call} differs from the oracle"
        assert np.array_equal(got.view(np.uint32), ws.view(np.uint32)), f"call {call} differs from the workspace entry"
    code = C.c_int(-1)
    assert qh.lib().qh_check_device_error(C.byref(code)) == 0
    assert code.value == 0


def test_noalloc_rejects_oversized_shape(qh, cuda):
    torch = cuda
    L = qh.lib()
    k, n_tok, out_f = 3584, 64, 8  # 64 rows of k=3584 need > 128 KiB of scratch
    w = torch.zeros(out_f * (k // 256) * 144, dtype=torch.uint8, device="cuda")
    x = torch.zeros((n_tok, k), dtype=torch.float32, device="cuda")
    out = torch.zeros((n_tok, out_f), dtype=torch.float32, device="cuda")
    rc = L.qh_matmul_q4k_f32_noalloc(C.c_void_p(w.data_ptr()), out_f, k, C.c_void_p(x.data_ptr()), n_tok,
                                     C.c_void_p(out.data_ptr()), None)
    assert rc == -5
    assert b"scratch" in L.qh_last_error()
