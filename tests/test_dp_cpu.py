# SPDX-License-Identifier: MIT
"""CPU (gloo, world size 2): the host side of the data-parallel plumbing --
the library communicator's id handed from rank 0 to every rank over a
torch.distributed group (qwen.haiku_b200.host.DataParallel; the NCCL
collectives themselves are tested on GPUs, tests/test_dp_gpu.py), bench.py's
max-over-ranks on a single rank, the reference arm's rank-0-only rule, and a
rank that leaves before the exchange -- without a GPU."""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from conftest import load_pkg
        qh = load_pkg()
        import ctypes as C
        got = []

        def exchange(b):  # what DataParallel.from_torch does, without creating the NCCL communicator
            obj = [b]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]
        if rank == 0:
            buf = (C.c_uint8 * 128)()
            qh.check(qh.lib().qh_dp_unique_id(buf), "qh_dp_unique_id")
            got = exchange(bytes(buf))
            assert got == bytes(buf)
        else:
            got = exchange(None)
        assert isinstance(got, bytes) and len(got) == 128 and any(got)
        ids = [None] * world
        dist.all_gather_object(ids, got)
        assert all(i == ids[0] for i in ids), "ranks received different ids"
        import bench
        assert bench.max_over_ranks(None, [1.0, 2.0]) == [1.0, 2.0]  # one rank: its own times
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging the peer
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_dp_collectives_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def test_reference_arm_only_rank0_works(monkeypatch):
    """Under torchrun the reference arm's non-zero ranks exit 0 at once."""
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setenv("RANK", "1")

    class Args:
        gpus, steps, warmup = 2, 1, 3
    assert bench.run_reference_arm(Args()) == 0


def _leaver(rank, world, port, q):
    """Rank 1 leaves before the communicator's id is handed out; rank 0's
    exchange must end with an error within the process group's short
    timeout instead of waiting for good."""
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import time
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    dist.barrier()
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the message is out before the process ends
        os._exit(0)  # leaves between steps: nothing of it is in flight
    t0 = time.monotonic()
    try:
        obj = [bytes(128)]
        dist.broadcast_object_list(obj, src=0)
        dist.barrier()
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_leaving_is_detected_by_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error after"), results[0]
    import re
    assert float(re.match(r"error after ([0-9.]+)s", results[0]).group(1)) < 30.0, results[0]
