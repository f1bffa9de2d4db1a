"""Failure handling of the tensor-parallel group, made on the host with gloo ranks on CPU:
a rank that leaves between steps is seen by the survivor before its next launch
(``TensorParallel.guard``), and a collective whose peer never joins ends with an error after
the group's timeout instead of blocking."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _departure_worker(rank, world, port, results):
    from linkq2_b200.runtime import parallel
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tp = parallel.init_from_env("gloo", timeout_s=3.0)
    x = torch.ones(4) * (rank + 1)
    tp.guard()                                   # step 1: everybody is there
    tp.all_reduce(x)
    assert x.tolist() == [3.0] * 4
    if rank == 1:
        tp.leave()                               # between steps, nothing in flight
        results[rank] = "left"
        return                                   # never joins another collective
    deadline = time.time() + 20
    while time.time() < deadline:                # the survivor's next steps
        try:
            tp.guard()
        except parallel.PeerLeft as e:
            results[rank] = f"stopped: {e}"
            break
        time.sleep(0.05)
    else:
        results[rank] = "never noticed"
        return
    # without the guard the library collective itself ends with an error after the timeout
    t0 = time.time()
    try:
        tp.all_reduce(torch.ones(4))
        results["timeout"] = "no error"
    except Exception as e:                       # gloo raises RuntimeError / DistBackendError
        results["timeout"] = f"{type(e).__name__} after {time.time() - t0:.1f}s"


def test_rank_leaves_between_steps():
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        results = manager.dict()
        ctx = mp.spawn(_departure_worker, args=(world, port, results), nprocs=world, join=False)
        t0 = time.time()
        while not ctx.join(timeout=1.0):
            assert time.time() - t0 < 60, "ranks did not finish"
        got = dict(results)
    assert got[1] == "left"
    assert got[0].startswith("stopped: rank(s) [1] left")
    assert "Error" in got["timeout"] and "no error" not in got["timeout"]


def test_guard_is_a_no_op_for_one_rank():
    from linkq2_b200.runtime import parallel
    tp = parallel.TensorParallel()
    tp.guard()
    tp.leave()
