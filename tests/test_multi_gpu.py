"""Row-sharded training on 2 GPUs gives the trees of a 1-GPU fit, bit for bit.

Histograms, left counts, the root count and the logloss are all-reduced as
exact int64 words (NCCL), so the engine is deterministic at any GPU count.
Skipped unless at least two CUDA devices are visible.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _ngpu():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_two_gpu_fit_equals_one_gpu(tmp_path):
    out = str(tmp_path / "two.npz")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29531", os.path.join(HERE, "multi_gpu_fit.py"), out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    two = np.load(out)
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "bsscl-gbm_b200"))
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M, datasets as D
    X, y = D.config3(n=25_000)
    m = M(n_estimators=12, max_depth=6, class_weight="balanced_sqrt", n_bins=255, random_state=3,
          verbose=False).fit(X[:20_000], y[:20_000])
    for t, tr in enumerate(m.trees):
        nc = tr[5]
        assert two["nc"][t] == nc, f"tree {t}"
        for i, k in [(0, "tf"), (1, "tt"), (2, "tv"), (3, "tl"), (4, "tr"), (6, "sg")]:
            assert np.array_equal(np.asarray(tr[i])[:nc], two[k][t][:nc]), f"tree {t} {k}"
    assert np.array_equal(m.predict_proba(X[20_000:]), two["proba"])
    assert np.allclose(np.array(m.train_loss_history_), two["loss"], rtol=1e-12, atol=0)
