"""Row-sharded training on 2 GPUs gives the trees of a 1-GPU fit, bit for bit:
best-first at depth 6, 8 and 12 (capped speculation, host replay with
on-demand expansion), depth-wise growth, NaN in every feature, the default
constructor's 257-bin features and the learned NaN direction.

Histograms (with the left counts and the root count in their count words),
the last level's totals and the logloss are all-reduced as exact int64 words
(NCCL), so the engine is deterministic at any GPU count.
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
def test_two_gpu_fits_equal_one_gpu(tmp_path):
    out = str(tmp_path / "two.npz")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29531", os.path.join(HERE, "multi_gpu_fit.py"), out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    two = np.load(out)
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "bsscl-gbm_b200"))
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    from multi_gpu_cases import CASES
    for name, (data, kw) in CASES.items():
        X, y, Xte = data()
        m = M(**kw).fit(X, y)
        assert len(m.trees) == len(two[f"{name}_nc"]), name
        for t, tr in enumerate(m.trees):
            nc = tr[5]
            assert two[f"{name}_nc"][t] == nc, f"{name} tree {t}"
            for i, k in [(0, "tf"), (1, "tt"), (2, "tv"), (3, "tl"), (4, "tr"), (6, "sg")]:
                assert np.array_equal(np.asarray(tr[i])[:nc], two[f"{name}_{k}"][t][:nc]), f"{name} tree {t} {k}"
        assert np.array_equal(m.predict_proba(Xte), two[f"{name}_proba"]), name
        assert np.allclose(np.array(m.train_loss_history_), two[f"{name}_loss"], rtol=1e-12, atol=0), name
