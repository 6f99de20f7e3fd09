"""Worker for test_multi_gpu: a rank of a row-sharded fit (run under torchrun).

Every rank fits config 3's data with the estimator (rows split across ranks,
histograms all-reduced exactly) and rank 0 saves the trees and predictions.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "bsscl-gbm_b200"))


def main(out_path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M, datasets as D
    X, y = D.config3(n=25_000)
    m = M(n_estimators=12, max_depth=6, class_weight="balanced_sqrt", n_bins=255, random_state=3,
          verbose=False)
    m.fit(X[:20_000], y[:20_000])
    proba = m.predict_proba(X[20_000:])
    if dist.get_rank() == 0:
        nc = np.array([t[5] for t in m.trees])
        cap = max(len(t[0]) for t in m.trees)
        arr = {k: np.stack([np.asarray(t[i]) for t in m.trees]) for i, k in
               [(0, "tf"), (1, "tt"), (2, "tv"), (3, "tl"), (4, "tr"), (6, "sg")]}
        np.savez(out_path, nc=nc, proba=proba, loss=np.array(m.train_loss_history_), **arr)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
