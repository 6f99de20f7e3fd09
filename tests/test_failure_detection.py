"""Failure detection, without faulting a GPU.

* On the GPU: the peer exchange's device-side wait has a time limit.  A wait
  for a signal that no rank sends runs out, reports GBM_ERR_TIMEOUT, and the
  device stays usable (the next kernel runs normally).
* On the host (gloo, two CPU processes): a rank that raises before a
  collective makes the other rank's collective end with an error within the
  process group's timeout instead of waiting for good.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

GBM_ERR_TIMEOUT = 6


@pytest.mark.gpu
def test_device_wait_runs_out_and_reports(engine):
    from bsscl_gbm_b200 import _lib
    L = _lib.lib()
    t0 = time.perf_counter()
    rc = L.gbm_test_peer_wait(0, 200)
    dt = time.perf_counter() - t0
    assert rc == GBM_ERR_TIMEOUT
    assert 0.15 < dt < 10.0
    # the context still works: a predict through the engine
    rng = np.random.default_rng(0)
    xb = rng.integers(0, 4, (1000, 3)).astype(np.uint8)
    packed = {"features": np.array([0, -1, -1], np.int16), "thresholds": np.array([1, 0, 0], np.int64),
              "values": np.array([0.0, -1.0, 1.0]), "left": np.array([1, -1, -1], np.int32),
              "right": np.array([2, -1, -1], np.int32), "offsets": np.array([0, 3], np.int32)}
    F, _ = engine.predict(xb, packed, 1, 1.0, 0.0)
    assert np.array_equal(F, np.where(xb[:, 0] <= 1, -1.0, 1.0))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, port, result):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=3))
    try:
        if rank == 1:
            raise RuntimeError("rank 1 leaves before the collective")
        t0 = time.perf_counter()
        try:
            dist.all_reduce(torch.ones(4))
            result[rank] = ("completed", time.perf_counter() - t0)
        except Exception as e:   # the peer is gone: the collective must fail, not hang
            result[rank] = (type(e).__name__, time.perf_counter() - t0)
    except RuntimeError:
        result[rank] = ("left", 0.0)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_that_leaves_ends_the_peer_collective_with_an_error():
    mgr = mp.Manager()
    result = mgr.dict()
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, port, result)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert result.get(1, ("?",))[0] == "left"
    status, dt = result.get(0, ("missing", 0.0))
    assert status not in ("completed", "missing")
    assert dt < 30.0
