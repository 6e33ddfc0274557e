# SPDX-License-Identifier: MIT
"""GPU: the library's data-parallel communicator (include/qh_dp.h, NCCL):
the per-step token gather, max-over-ranks of timings, and a rank that leaves
between steps. One rank on one GPU always; two ranks (child processes, one
GPU each) when two GPUs are visible. NVLS is off in every child
(NCCL_NVLS_ENABLE=0) and the leaving rank has nothing in flight when it
exits; the survivor's bounded wait aborts its communicator."""
import ctypes as C
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_one_rank_gather_and_max(qh, cuda):
    torch = cuda
    dp = qh.host.DataParallel(0, 1, lambda b: b, timeout_ms=5000)
    local = torch.arange(7, dtype=torch.int32, device="cuda") + 40
    out = torch.full((7,), -1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    dp.gather(local.data_ptr(), 7, out.data_ptr(), s)
    dp.wait(s)
    assert torch.equal(out, local)
    assert dp.max([1.5, -2.0]) == [1.5, -2.0]
    dp.close()


def _child(rank, world, id_path, mode, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import time
    import torch
    from conftest import load_pkg
    try:
        torch.cuda.set_device(rank)
        qh = load_pkg()
        qh.check(qh.lib().qh_set_device(rank), "qh_set_device")

        def exchange(b):  # rank 0 writes the id, the others wait for the file
            if b is not None:
                with open(id_path + ".tmp", "wb") as f:
                    f.write(b)
                os.replace(id_path + ".tmp", id_path)
                return b
            for _ in range(600):
                if os.path.exists(id_path):
                    return open(id_path, "rb").read()
                time.sleep(0.05)
            raise TimeoutError("no id")
        dp = qh.host.DataParallel(rank, world, exchange, timeout_ms=3000)
        B = 5
        s = torch.cuda.current_stream().cuda_stream
        out = torch.empty(world * B, dtype=torch.int32, device="cuda")
        steps = 3 if mode == "ok" else 1
        for step in range(steps):
            local = torch.arange(B, dtype=torch.int32, device="cuda") + 100 * rank + 1000 * step
            dp.gather(local.data_ptr(), B, out.data_ptr(), s)
            dp.wait(s)
            want = torch.cat([torch.arange(B, dtype=torch.int32) + 100 * r + 1000 * step for r in range(world)])
            assert torch.equal(out.cpu(), want), (out, want)
        if mode == "ok":
            assert dp.max([1.0 + rank, 10.0 - rank]) == [float(world), 10.0]
            dp.close()
            q.put((rank, "ok"))
            return
        if rank == 1:  # leaves between steps: its gather is complete, nothing in flight
            q.put((rank, "left"))
            return
        t0 = time.monotonic()
        try:
            local = torch.zeros(B, dtype=torch.int32, device="cuda")
            dp.gather(local.data_ptr(), B, out.data_ptr(), s)
            dp.wait(s)
            q.put((rank, "no error"))
        except qh.QHError as e:
            q.put((rank, f"error after {time.monotonic() - t0:.1f}s: status {e.status}"))
    except Exception as e:
        q.put((rank, repr(e)))


def _run_two(mode, tmp_path):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    id_path = str(tmp_path / f"nccl_id_{mode}")
    procs = [ctx.Process(target=_child, args=(r, 2, id_path, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def _two_gpus():
    import torch
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_two_ranks_gather_and_max(qh, cuda, tmp_path):
    assert _run_two("ok", tmp_path) == {0: "ok", 1: "ok"}


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_rank_leaving_ends_the_next_gather_with_an_error(qh, cuda, tmp_path):
    res = _run_two("leave", tmp_path)
    assert res[1] == "left"
    assert res[0].startswith("error after") and res[0].endswith("status -6"), res[0]
    import re
    assert float(re.match(r"error after ([0-9.]+)s", res[0]).group(1)) < 30.0, res[0]
