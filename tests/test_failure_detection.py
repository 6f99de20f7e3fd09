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


_LONELY_RANK = r"""
import sys, time
import numpy as np
sys.path.insert(0, sys.argv[1])
from bsscl_gbm_b200 import Engine
eng = Engine(0)
uid = Engine.nccl_unique_id()
t0 = time.perf_counter()
try:
    eng.init_comm(uid, 2, 0, timeout_ms=1500)      # rank 1 never joins
    print("JOINED")
except RuntimeError as e:
    print("ERR", time.perf_counter() - t0, str(e).replace("\n", " "))
xb = np.zeros((100, 2), np.uint8)
packed = {"features": np.array([-1], np.int16), "thresholds": np.array([0], np.int64),
          "values": np.array([0.5]), "left": np.array([-1], np.int32), "right": np.array([-1], np.int32),
          "offsets": np.array([0, 1], np.int32)}
F, _ = eng.predict(xb, packed, 1, 2.0, 0.0)
print("PREDICT", float(F[0]))
eng.close()
"""


@pytest.mark.gpu
def test_communicator_whose_peer_never_joins_times_out():
    """gbm_ctx_init_comm for a 2-rank world with only rank 0 present: the
    non-blocking NCCL init is polled with the engine's time limit, runs out,
    is aborted and reported as GBM_ERR_TIMEOUT, and the context still runs
    kernels afterwards.  A child process (NVLS off) so that nothing of the
    aborted communicator outlives the test."""
    import subprocess
    import sys
    from conftest import ROOT
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    out = subprocess.run([sys.executable, "-c", _LONELY_RANK, os.path.join(ROOT, "bsscl-gbm_b200")], env=env,
                         capture_output=True, text=True, timeout=180)
    lines = out.stdout.strip().splitlines()
    err = [ln for ln in lines if ln.startswith("ERR")]
    assert err, out.stdout + out.stderr
    dt = float(err[0].split()[1])
    assert "timeout" in err[0] and 1.0 < dt < 60.0, err[0]
    assert "PREDICT 1.0" in lines, out.stdout + out.stderr
