# SPDX-License-Identifier: MIT
"""GPU: the device expf/logf (qwen.haiku_b200/csrc/qh_libm.cuh) against the
host C library's expf/logf -- the functions the reference calls -- on all
2^32 float bit patterns. Bar: identical bits (any NaN equals any NaN).

The model's per-layer Q8_K re-quantization turns a single one-ulp
difference in a SiLU or softmax into different greedy tokens after tens of
steps, so these two functions must be the reference's, not merely accurate.
"""
import platform

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CHUNK = 1 << 28


@pytest.mark.parametrize("fn,name", [(0, "expf"), (1, "logf")])
def test_device_libm_equals_host_on_all_inputs(qh, cuda, oracle, fn, name):
    import ctypes as C
    torch = cuda
    L = qh.lib()
    dev = torch.empty(CHUNK, dtype=torch.float32, device="cuda")
    host = torch.empty(CHUNK, dtype=torch.float32, pin_memory=True)
    s = torch.cuda.current_stream()
    total, first_bad = 0, None
    for first in range(0, 1 << 32, CHUNK):
        qh.check(L.qh_libm_eval(fn, first, CHUNK, C.c_void_p(dev.data_ptr()), C.c_void_p(s.cuda_stream)),
                 "qh_libm_eval")
        host.copy_(dev, non_blocking=True)
        s.synchronize()
        n, bad = oracle.libm_mismatches(fn, first, host.numpy())
        total += n
        if bad is not None and first_bad is None:
            first_bad = bad
    print(f"{name}: {total} of 2^32 inputs differ from the host library ({platform.libc_ver()})")
    assert total == 0, f"{name}: {total} inputs differ, first at bit pattern {first_bad:#010x}"


def test_libm_eval_rejects_bad_arguments(qh, cuda):
    L = qh.lib()
    assert L.qh_libm_eval(2, 0, 16, None, None) == -1  # QH_ERR_INVALID: unknown function
