"""Worker for test_multi_gpu: a rank of row-sharded fits (run under torchrun).

Every rank fits each case's data with the estimator (rows split across
ranks, histograms all-reduced exactly) and rank 0 saves the trees and
predictions of every case.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "bsscl-gbm_b200"))
sys.path.insert(0, HERE)


def main(out_path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    from multi_gpu_cases import CASES
    out = {}
    for name, (data, kw) in CASES.items():
        X, y, Xte = data()
        m = M(**kw).fit(X, y)
        proba = m.predict_proba(Xte)
        if dist.get_rank() == 0:
            out[f"{name}_nc"] = np.array([t[5] for t in m.trees])
            for i, k in [(0, "tf"), (1, "tt"), (2, "tv"), (3, "tl"), (4, "tr"), (6, "sg")]:
                out[f"{name}_{k}"] = np.stack([np.asarray(t[i]) for t in m.trees])
            out[f"{name}_proba"] = proba
            out[f"{name}_loss"] = np.array(m.train_loss_history_)
    if dist.get_rank() == 0:
        np.savez(out_path, **out)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
