"""Record the reference's own fits at the benchmark configurations' full sizes.

Run once, in a container where the reference package is importable (the
oracle library must be built: ``make -C oracle``):

    PYTHONPATH=<reference>/src NUMBA_CACHE_DIR=/tmp/numba_cache \
        python tests/golden/make_golden_full.py <reference>/src [case ...]

Cases (every one uses the seeded generators of ``bsscl_gbm_b200.datasets``;
no feature matrix is stored, the tests regenerate it):

* ``cfg4_d6``  config 4, 1,000,000 x 100 float32 with 30 % NaN, max_depth 6,
  205 trees: the benchmark's workload (its 5 warm-up + 200 timed rounds).
* ``cfg4_d8``  the same data at max_depth 8, 200 trees (configs[3] literally).
* ``cfg2``     config 2 at its full 284,807 x 30, balanced_sqrt, 500 trees.
* ``cfg3``     config 3 at its full 50,000 x 20, balanced_sqrt, 300 trees.
* ``top257``   the reference's default constructor (n_bins 'auto' = 256 at
  p = 30, so every feature has 257 bin ids) on ``datasets.top_bin``, 30
  trees: splits at threshold 255, bin 256 alone on the right.

Each file ``fit_full_<case>.npz`` holds the reference's trees, train-loss
history, base score, bin edges / counts / NaN bins, a hash of its uint16 bin
matrix, per-round hashes of its row and feature samples, its predict_proba on
a held-out slice, and -- computed here with the CPU oracle (test
infrastructure) -- the trajectory of the engine's exact fixed-point
arithmetic (``exact_*``: trees and losses of the oracle's EXACT mode with the
engine's fixed-point exponent) together with an audit of the first node
where that trajectory leaves the reference's: both splits evaluated in exact
rational arithmetic on the reference's own round inputs.
"""

from __future__ import annotations

import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for _p in (os.path.join(REPO, "bsscl-gbm_b200"), os.path.join(REPO, "oracle")):
    sys.path.insert(0, _p)

TREE_KEYS = (("tf", -1, np.int32), ("tt", 0, np.int64), ("tv", 0.0, np.float64),
             ("tl", -1, np.int32), ("tr", -1, np.int32), ("sg", 0.0, np.float64))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def tree_arrays(trees, prefix=""):
    T = len(trees)
    maxn = max(len(t[0]) for t in trees)
    arr = {prefix + k: np.full((T, maxn), fill, dtype=dt) for k, fill, dt in TREE_KEYS}
    ncs = np.zeros(T, dtype=np.int32)
    for t, tr in enumerate(trees):
        for (k, _, _), a in zip(TREE_KEYS, (tr[0], tr[1], tr[2], tr[3], tr[4], tr[6])):
            arr[prefix + k][t, :len(a)] = a
        ncs[t] = tr[5]
    arr[prefix + "nc"] = ncs
    return arr


def engine_scale_bits(wmax, chunk=16384):
    """The engine's fixed-point exponent (libgbm_b200): 62 - ceil(log2(chunk * max(1, wmax)))."""
    return 62 - int(np.ceil(np.log2(chunk * max(1.0, wmax))))


CASES = {
    "cfg4_d6": dict(data="config4", n_estimators=205, max_depth=6, n_bins=255, random_state=0),
    "cfg4_d8": dict(data="config4", n_estimators=200, max_depth=8, n_bins=255, random_state=0),
    "cfg2": dict(data="config2", n_estimators=500, max_depth=6, class_weight="balanced_sqrt", n_bins=255,
                 random_state=0),
    "cfg3": dict(data="config3", n_estimators=300, max_depth=6, class_weight="balanced_sqrt", n_bins=255,
                 random_state=0),
    "top257": dict(data="top_bin", n_estimators=30, random_state=0),
}


def case_data(D, which):
    """(X_train, y_train, X_heldout) for a case; the held-out rows are a
    second seeded draw of the same generator (same feature distributions)."""
    if which == "config4":
        X, y = D.config4(n=1_000_000)
        Xh, _ = D.config4(n=20_000, seed=13)
    elif which == "top_bin":
        X, y = D.top_bin()
        Xh, _ = D.top_bin(n=5_000, seed=22)
    elif which == "config2":
        X, y = D.config2()
        Xh, _ = D.config2(n=20_000, seed=11, n_pos=40)
    else:
        X, y = D.config3()
        Xh, _ = D.config3(n=20_000, seed=12)
    return X, y, Xh


def run_case(E, D, O, A, name):
    spec = dict(CASES[name])
    which = spec.pop("data")
    X, y, Xh = case_data(D, which)
    captured = []
    cls = E.HybridHistGBMNumbaV1_0_1
    orig = cls._build_one_tree

    def spy(self, X_bin, grad, hess, sample_idx, feat_idx, n_features):
        tree = orig(self, X_bin, grad, hess, sample_idx, feat_idx, n_features)
        captured.append((grad.copy(), hess.copy(), sample_idx.copy(), feat_idx.copy()))
        return tree

    t0 = time.perf_counter()
    cls._build_one_tree = spy
    try:
        m = cls(verbose=False, **spec)
        m.fit(X, y)
    finally:
        cls._build_one_tree = orig
    t_ref = time.perf_counter() - t0
    Xb, _ = m._bin_features(X)
    Xb = np.ascontiguousarray(Xb)
    ref = [tuple(t) for t in m.trees]
    proba_held = m.predict_proba(Xh)
    # the engine's arithmetic on the same bins: the oracle's EXACT mode
    w2 = O.class_weights(y, spec.get("class_weight", "balanced_sqrt"))
    S = engine_scale_bits(float(np.max(w2)))
    t1 = time.perf_counter()
    ex = O.fit_binary(Xb, y, m.feature_bin_counts, n_estimators=len(ref), learning_rate=m.learning_rate,
                      max_leaves=m.max_leaves, max_depth=m.max_depth, min_samples_leaf=m.min_samples_leaf,
                      min_child_weight=m.min_child_weight, reg_lambda=m.reg_lambda, gamma=m.gamma,
                      subsample=m.subsample, colsample=m.colsample_bytree,
                      class_weight=spec.get("class_weight", "balanced_sqrt"), random_state=spec["random_state"],
                      mode=O.MODE_EXACT, scale_bits=S)
    t_exact = time.perf_counter() - t1
    div = A.first_divergence(ref, ex["trees"])
    audit = {"kind": "none", "rel_gap": 0.0, "n_rows": 0}
    if div is not None:
        t, node = div
        g, h, s, _ = captured[t]
        res = A.audit_node(Xb, g, h, s, m.feature_bin_counts, ref[t], ex["trees"][t], node,
                           float(m.reg_lambda), float(m.min_child_weight))
        audit = {"kind": res.get("kind"), "rel_gap": float(res.get("rel_gap", 0.0)),
                 "n_rows": int(res.get("n_rows", 0))}
    extra = {}
    if div is not None:
        extra = dict(div_tree=div[0], div_node=div[1])
    np.savez_compressed(
        os.path.join(HERE, f"fit_full_{name}.npz"),
        params=np.array(repr(CASES[name])), n_trees=len(ref), **tree_arrays(ref),
        **tree_arrays(ex["trees"], "exact_"), exact_train_loss=ex["train_loss"], exact_scale_bits=S,
        base_score=m.base_score_, learning_rate=m.learning_rate, max_leaves=m.max_leaves,
        max_depth=m.max_depth, min_child_weight=m.min_child_weight, subsample=m.subsample,
        colsample=m.colsample_bytree, reg_lambda=m.reg_lambda, gamma=m.gamma,
        min_samples_leaf=m.min_samples_leaf, binning_strategy=m.binning_strategy, n_bins=m.n_bins,
        edges=m.bin_edges, counts=m.feature_bin_counts, nan_bin_id=m._nan_bin_id, max_bins=m._max_bins,
        X_bin_sha=sha(Xb.astype(np.uint16)), train_loss=np.array(m.train_loss_history_),
        proba_heldout=proba_held, proba_train_head=m.predict_proba(X[:20_000]),
        sample_sha=np.array([sha(c[2]) for c in captured]), feat_sha=np.array([sha(c[3]) for c in captured]),
        audit_kind=np.array(audit["kind"]), audit_rel_gap=audit["rel_gap"], audit_rows=audit["n_rows"],
        has_div=div is not None, ref_seconds=t_ref, exact_seconds=t_exact, **extra)
    print(f"{name}: {len(ref)} trees, ref {t_ref:.1f} s, exact {t_exact:.1f} s, divergence {div}, "
          f"audit {audit}", flush=True)


def main(ref_src, names):
    sys.path.insert(0, ref_src)
    import bsscl_gbm.estimator_v1_0_1 as E
    from bsscl_gbm_b200 import datasets as D
    import audit as A
    import oracle as O
    for name in names or list(CASES):
        run_case(E, D, O, A, name)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden_full.py <reference>/src [" + "|".join(CASES) + " ...]")
    main(sys.argv[1], sys.argv[2:])
