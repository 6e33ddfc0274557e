# SPDX-License-Identifier: MIT
"""GPU: the kernels' bounded-wait timeout path, without a fault. A grouped
matvec plan leaves out every copy of one tile (qh_matvec_plan_test_timeout)
with a short poll limit: the consumers' wait for that stage runs out, the
CTA records the timeout in the device error word, drains its own copies in
flight and returns; qh_check_device_error reports QH_ERR_DEVICE (code 1)
and clears the word; the context stays usable -- the same plan without the
hook gives outputs bit-identical to the oracle and a clean check."""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q4_K = 12


@pytest.mark.parametrize("tile", [0, 5])
def test_withheld_copy_times_out_and_reports(qh, cuda, oracle, tile):
    torch = cuda
    h, L = qh.host, qh.lib()
    k, out_f = 1024, 3072
    w_np = h.synth_blocks(Q4_K, out_f * (k // 256), 0x71E0 + tile)
    x_np = h.synth_normal(k, 0x71E1 + tile).reshape(1, k)
    w, x = h.to_device(w_np), h.to_device(x_np)
    xq = h.quantize_q8k(x, k, 1)
    out = torch.zeros((1, out_f), dtype=torch.float32, device="cuda")
    plan = h.MatvecPlan(Q4_K, [(w, xq, out, k, out_f)], 1)
    code = C.c_int(-1)
    torch.cuda.synchronize()
    assert L.qh_check_device_error(C.byref(code)) == 0
    qh.check(L.qh_matvec_plan_test_timeout(plan.handle, tile, 2000), "qh_matvec_plan_test_timeout")
    t0 = time.monotonic()
    plan.run()
    torch.cuda.synchronize()  # returns: every wait was bounded
    took = time.monotonic() - t0
    rc = L.qh_check_device_error(C.byref(code))
    assert rc == -6 and code.value == 1, (rc, code.value)  # QH_ERR_DEVICE, kDevWaitTimeout
    assert b"timed out" in L.qh_last_error()
    assert took < 10.0, f"the bounded waits took {took:.1f} s"
    assert L.qh_check_device_error(C.byref(code)) == 0 and code.value == 0  # cleared
    # the context is usable: the same plan without the hook is exact
    qh.check(L.qh_matvec_plan_test_timeout(plan.handle, -1, 0), "qh_matvec_plan_test_timeout")
    plan.run()
    torch.cuda.synchronize()
    want = oracle.matmul(Q4_K, w_np, out_f, k, x_np).reshape(1, out_f)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert L.qh_check_device_error(C.byref(code)) == 0
    plan.close() if hasattr(plan, "close") else None


def test_hook_rejects_a_tile_outside_the_plan(qh, cuda):
    torch = cuda
    h, L = qh.host, qh.lib()
    k, out_f = 256, 64
    w = h.to_device(h.synth_blocks(Q4_K, out_f, 3))
    xq = h.quantize_q8k(h.to_device(h.synth_normal(k, 4).reshape(1, k)), k, 1)
    out = torch.zeros((1, out_f), dtype=torch.float32, device="cuda")
    plan = h.MatvecPlan(Q4_K, [(w, xq, out, k, out_f)], 1)
    assert L.qh_matvec_plan_test_timeout(plan.handle, 1 << 20, 10) == -1
