"""Failure detection on the host (no GPU): ranks that never join or die between steps.

Faults are made on the host, as gloo ranks on CPU: a missing rank must make the
others fail within the process-group timeout instead of hanging, and a rank
that raises must surface as an error on its peers' next collective.
"""

import multiprocessing as mp
import os
import socket
import time


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _join_alone(port, box):
    os.environ["TORCH_DISTRIBUTED_TIMEOUT_MINUTES"] = "0.05"  # 3 s
    from uno_b200.parallel.state import init_tp

    t0 = time.time()
    try:
        init_tp(2, 0, backend="gloo", init_method=f"tcp://127.0.0.1:{port}")
        box.put(("joined", time.time() - t0))
    except Exception as exc:  # the peer never arrives
        box.put(("error", time.time() - t0, type(exc).__name__))


def test_rank_that_never_joins_times_out():
    ctx = mp.get_context("spawn")
    box = ctx.Queue()
    p = ctx.Process(target=_join_alone, args=(_port(), box))
    p.start()
    out = box.get(timeout=120)
    p.join(30)
    assert out[0] == "error" and out[1] < 60, out


def _step_worker(rank, port, box):
    import torch
    import torch.distributed as dist

    from uno_b200.parallel.state import init_tp

    os.environ["TORCH_DISTRIBUTED_TIMEOUT_MINUTES"] = "0.1"  # 6 s
    init_tp(2, rank, backend="gloo", init_method=f"tcp://127.0.0.1:{port}")
    x = torch.ones(4)
    dist.all_reduce(x)  # step 1: both ranks healthy
    if rank == 1:
        os._exit(3)  # dies between steps, with nothing in flight
    t0 = time.time()
    try:
        dist.all_reduce(x)  # step 2: the peer is gone
        box.put(("completed", time.time() - t0))
    except Exception as exc:
        box.put(("error", time.time() - t0, type(exc).__name__))


def test_peer_that_dies_between_steps_fails_the_next_collective():
    ctx = mp.get_context("spawn")
    box = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_step_worker, args=(r, port, box)) for r in range(2)]
    for p in procs:
        p.start()
    out = box.get(timeout=180)
    for p in procs:
        p.join(30)
    assert procs[1].exitcode == 3
    assert out[0] == "error" and out[1] < 90, out


def test_engine_follower_failure_is_reported():
    """A TP follower that raises logs its traceback and re-raises (``worker_main``)."""
    import pytest

    from uno_b200.engine import worker

    class _Cfg:
        tensor_parallel_size = 1
        device = "cpu"

    called = {}

    def boom(*a, **k):
        called["init"] = True
        raise RuntimeError("init failed")

    orig = worker.init_distributed
    worker.init_distributed = boom
    try:
        with pytest.raises(RuntimeError, match="init failed"):
            worker.worker_main(_Cfg(), 1, 0)
    finally:
        worker.init_distributed = orig
    assert called["init"]
