"""Calibrate the CPU port (oracle.c, REF mode) against the reference itself.

TEST INFRASTRUCTURE ONLY.  bench.py's reference arm times the port, because
the reference (Python + Numba) cannot travel to the GPU box.  This script,
run where the reference is importable, times both on the same rows, the same
parameters and the same host threads, so the port's rounds/s can be read as
the reference's:

    PYTHONPATH=<reference>/src NUMBA_CACHE_DIR=/tmp/numba_cache \
        python oracle/calibrate_port.py <reference>/src [rows] [trees]

Workload: config 4's data (seeded stand-in, 1M x 100 float32, 30 % NaN) cut
to `rows` rows, binned by the reference, trained at bench.py's parameters
(depth 6, 63 leaves, lr 0.08, subsample 0.75, colsample 0.7, mcw 3,
balanced_sqrt).  The reference is warmed up (JIT) on the same dtypes first;
its rounds/s is n_estimators / times['training'] (E:3226-3240).  Prints one
JSON line.
"""
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(REPO, "bsscl-gbm_b200"))
sys.path.insert(0, HERE)


def main(ref_src, rows=200_000, trees=20):
    sys.path.insert(0, ref_src)
    import numba
    import bsscl_gbm.estimator_v1_0_1 as E
    import oracle as O
    from bsscl_gbm_b200 import datasets as D
    X, y = D.config4(n=rows)
    params = dict(max_depth=6, learning_rate=0.08, n_bins=255, min_child_weight=3.0, subsample=0.75,
                  colsample_bytree=0.7, class_weight="balanced_sqrt", random_state=0, verbose=False)
    E.HybridHistGBMNumbaV1_0_1(n_estimators=2, **params).fit(X[:20_000], y[:20_000])   # JIT warm-up
    m = E.HybridHistGBMNumbaV1_0_1(n_estimators=trees, **params)
    m.fit(X, y)
    ref_rps = trees / (m.times["training"] / 1000.0)
    Xb, _ = m._bin_features(X)
    kw = dict(learning_rate=m.learning_rate, max_leaves=m.max_leaves, max_depth=m.max_depth,
              min_samples_leaf=m.min_samples_leaf, min_child_weight=m.min_child_weight,
              reg_lambda=m.reg_lambda, gamma=m.gamma, subsample=m.subsample, colsample=m.colsample_bytree,
              class_weight="balanced_sqrt", random_state=0, mode=O.MODE_REF)
    O.fit_binary(Xb, y, m.feature_bin_counts, n_estimators=1, **kw)
    t0 = time.perf_counter()
    res = O.fit_binary(Xb, y, m.feature_bin_counts, n_estimators=trees, **kw)
    port_rps = trees / (time.perf_counter() - t0)
    same = all(np.array_equal(a[0][:a[5]], b[0][:b[5]]) and np.array_equal(a[1][:a[5]], b[1][:b[5]])
               for a, b in zip(res["trees"], m.trees))
    print(json.dumps({"rows": rows, "features": int(X.shape[1]), "trees": trees,
                      "reference_rounds_per_s": ref_rps, "port_rounds_per_s": port_rps,
                      "port_over_reference": port_rps / ref_rps, "numba_threads": numba.get_num_threads(),
                      "port_threads": O.num_threads(), "cpu_count": os.cpu_count(),
                      "same_topology": bool(same)}))


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: calibrate_port.py <reference>/src [rows] [trees]")
    main(sys.argv[1], *(int(a) for a in sys.argv[2:4]))
