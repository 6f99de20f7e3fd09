"""Generate the golden fixtures in this directory by running the reference.

Run once, in a container where the reference package is importable:

    PYTHONPATH=<reference>/src NUMBA_CACHE_DIR=/tmp/numba_cache \
        python tests/golden/make_golden.py <reference>/src

It imports ``bsscl_gbm.estimator_v1_0_1`` (the reference's Numba CPU path),
calls its binning, tree builders, predict kernels, NumPy ``RandomState``
sampler and full ``fit`` on seeded synthetic inputs, and writes compressed
``.npz`` files next to this script.  The tests never import the reference:
they compare the oracle (and, on a GPU, the CUDA engine) against these files.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "bsscl-gbm_b200"))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def model_json_case(E, D):
    """A reference fit saved with its own save_model (E:4035-4107), plus the
    reference's predict_proba before and after its own load_model."""
    X, y = D.config3(n=25_000)
    m = E.HybridHistGBMNumbaV1_0_1(n_estimators=12, max_depth=6, learning_rate=0.1,
                                   class_weight="balanced_sqrt", n_bins=255, random_state=0,
                                   verbose=False)
    m.fit(X[:20_000], y[:20_000])
    path = os.path.join(HERE, "model_ref_cfg3.json")
    m.save_model(path)
    back = E.HybridHistGBMNumbaV1_0_1.load_model(path)
    np.savez_compressed(os.path.join(HERE, "model_ref_cfg3.npz"),
                        proba_test=m.predict_proba(X[20_000:]),
                        proba_test_loaded=back.predict_proba(X[20_000:]))
    return {"model_ref_cfg3": (len(m.trees),)}


def multiclass_case(E, D):
    """A reference multi-class fit (E:2949-3065): its trees per class, its
    predict_proba, train losses, and the first rounds' gradients, sample and
    features (for tie audits)."""
    X, y = D.multiclass()
    Xtr, ytr, Xte = X[:6_400], y[:6_400], X[6_400:]
    params = dict(n_estimators=10, max_depth=5, learning_rate=0.1, n_bins=64,
                  class_weight="balanced_sqrt", random_state=0)
    captured = []
    cls = E.HybridHistGBMNumbaV1_0_1
    orig = cls._build_one_tree

    def spy(self, X_bin, grad, hess, sample_idx, feat_idx, n_features):
        captured.append((grad.copy(), hess.copy(), sample_idx.copy(), feat_idx.copy()))
        return orig(self, X_bin, grad, hess, sample_idx, feat_idx, n_features)

    cls._build_one_tree = spy
    try:
        m = cls(verbose=False, **params)
        m.fit(Xtr, ytr)
    finally:
        cls._build_one_tree = orig
    K = m.n_classes_
    T = len(m.mc_trees[0])
    maxn = max(len(t[0]) for ts in m.mc_trees for t in ts)
    arr = {k: np.full((K, T, maxn), fill, dtype=dt) for k, fill, dt in [
        ("tf", -1, np.int32), ("tt", 0, np.int64), ("tv", 0.0, np.float64),
        ("tl", -1, np.int32), ("tr", -1, np.int32), ("sg", 0.0, np.float64)]}
    ncs = np.zeros((K, T), dtype=np.int32)
    for k in range(K):
        for t, (tf, tt, tv, tl, tr, nc, sg) in enumerate(m.mc_trees[k]):
            for key, a in zip(("tf", "tt", "tv", "tl", "tr", "sg"), (tf, tt, tv, tl, tr, sg)):
                arr[key][k, t, :len(a)] = a
            ncs[k, t] = nc
    extra = {}
    for r_ in range(min(3, T)):
        for k in range(K):
            g, h, s, f = captured[r_ * K + k]
            extra[f"r{r_}_k{k}_g"] = g
            extra[f"r{r_}_k{k}_h"] = h
        extra[f"r{r_}_sample"] = captured[r_ * K][2]
        extra[f"r{r_}_feat"] = captured[r_ * K][3]
    Xb, _ = m._bin_features(Xtr)
    np.savez_compressed(
        os.path.join(HERE, "fit_mc.npz"), params=np.array(repr(params)), n_classes=K, n_trees=T, nc=ncs,
        **arr, **extra, learning_rate=m.learning_rate, max_leaves=m.max_leaves, max_depth=m.max_depth,
        min_child_weight=m.min_child_weight, subsample=m.subsample, colsample=m.colsample_bytree,
        reg_lambda=m.reg_lambda, gamma=m.gamma, min_samples_leaf=m.min_samples_leaf, n_bins=m.n_bins,
        edges=m.bin_edges, counts=m.feature_bin_counts, nan_bin_id=m._nan_bin_id,
        X_bin_sha=sha(Xb.astype(np.uint16)), train_loss=np.array(m.train_loss_history_),
        proba_test=m.predict_proba(Xte), sample_sha=np.array([sha(c[2]) for c in captured[::K]]))
    return {"fit_mc": (K, T)}


def regression_case(E, D, loss):
    """A reference regression fit (E:2607-2705) with its own Regressor class:
    trees, predictions, train losses, the first rounds' gradients and samples."""
    X, y = D.regression()
    Xtr, ytr, Xte = X[:6_400], y[:6_400], X[6_400:]
    params = dict(n_estimators=10, max_depth=5, learning_rate=0.1, n_bins=64, random_state=0, loss=loss)
    captured = []
    cls = E.HybridHistGBMNumbaV1_0_1
    orig = cls._build_one_tree

    def spy(self, X_bin, grad, hess, sample_idx, feat_idx, n_features):
        captured.append((grad.copy(), hess.copy(), sample_idx.copy(), feat_idx.copy()))
        return orig(self, X_bin, grad, hess, sample_idx, feat_idx, n_features)

    cls._build_one_tree = spy
    try:
        m = E.HybridHistGBMRegressorV1_0_1(verbose=False, **params)
        m.fit(Xtr, ytr)
    finally:
        cls._build_one_tree = orig
    T = len(m.trees)
    maxn = max(len(t[0]) for t in m.trees)
    arr = {k: np.full((T, maxn), fill, dtype=dt) for k, fill, dt in [
        ("tf", -1, np.int32), ("tt", 0, np.int64), ("tv", 0.0, np.float64),
        ("tl", -1, np.int32), ("tr", -1, np.int32), ("sg", 0.0, np.float64)]}
    ncs = np.zeros(T, dtype=np.int32)
    for t, (tf, tt, tv, tl, tr, nc, sg) in enumerate(m.trees):
        for key, a in zip(("tf", "tt", "tv", "tl", "tr", "sg"), (tf, tt, tv, tl, tr, sg)):
            arr[key][t, :len(a)] = a
        ncs[t] = nc
    extra = {}
    for r_ in range(min(3, T)):
        g, h, s, f = captured[r_]
        extra[f"r{r_}_g"], extra[f"r{r_}_h"], extra[f"r{r_}_sample"], extra[f"r{r_}_feat"] = g, h, s, f
    Xb, _ = m._bin_features(Xtr)
    np.savez_compressed(
        os.path.join(HERE, f"fit_reg_{loss}.npz"), params=np.array(repr(params)), n_trees=T, nc=ncs, **arr,
        **extra, init_score=m.init_score_, learning_rate=m.learning_rate, max_leaves=m.max_leaves,
        max_depth=m.max_depth, min_child_weight=m.min_child_weight, subsample=m.subsample,
        colsample=m.colsample_bytree, reg_lambda=m.reg_lambda, gamma=m.gamma,
        min_samples_leaf=m.min_samples_leaf, n_bins=m.n_bins, edges=m.bin_edges, counts=m.feature_bin_counts,
        nan_bin_id=m._nan_bin_id, X_bin_sha=sha(Xb.astype(np.uint16)), train_loss=np.array(m.train_loss_history_),
        pred_test=m.predict(Xte), sample_sha=np.array([sha(c[2]) for c in captured]))
    return {f"fit_reg_{loss}": (T,)}


def monotone_case(E, D):
    """A fit of config 1's data (first 3000 rows) with monotone constraints
    on four features: the reference's trees after post-prune and the
    monotone clip (E:2450-2457), its train loss and predict_proba."""
    Xtr, ytr, Xte, _ = D.config1()
    X, y = Xtr[:3000], ytr[:3000]
    mono = [0] * X.shape[1]
    mono[0], mono[1], mono[4], mono[7] = 1, -1, 1, -1
    params = dict(n_estimators=20, max_depth=4, learning_rate=0.1, n_bins=64, class_weight=None,
                  random_state=5, monotone_constraints=mono)
    m = E.HybridHistGBMNumbaV1_0_1(verbose=False, **params)
    m.fit(X, y)
    T = len(m.trees)
    maxn = max(len(t[0]) for t in m.trees)
    arr = {k: np.full((T, maxn), fill, dtype=dt) for k, fill, dt in [
        ("tf", -1, np.int32), ("tt", 0, np.int64), ("tv", 0.0, np.float64),
        ("tl", -1, np.int32), ("tr", -1, np.int32), ("sg", 0.0, np.float64)]}
    ncs = np.zeros(T, dtype=np.int32)
    for t, (tf, tt, tv, tl, tr, nc, sg) in enumerate(m.trees):
        for k, a in zip(("tf", "tt", "tv", "tl", "tr", "sg"), (tf, tt, tv, tl, tr, sg)):
            arr[k][t, :len(a)] = a
        ncs[t] = nc
    np.savez_compressed(
        os.path.join(HERE, "fit_mono.npz"), params=np.array(repr(params)), n_trees=T, nc=ncs, **arr,
        mono=np.array(mono, dtype=np.int32), base_score=m.base_score_, learning_rate=m.learning_rate,
        max_leaves=m.max_leaves, max_depth=m.max_depth, min_child_weight=m.min_child_weight,
        subsample=m.subsample, colsample=m.colsample_bytree, reg_lambda=m.reg_lambda, gamma=m.gamma,
        min_samples_leaf=m.min_samples_leaf, n_bins=m.n_bins, binning_strategy=m.binning_strategy,
        edges=m.bin_edges, counts=m.feature_bin_counts, nan_bin_id=m._nan_bin_id,
        train_loss=np.array(m.train_loss_history_),
        proba_test=m.predict_proba(Xte))
    return {"fit_mono": (T, int(ncs.sum()))}


def early_stop_case(E, D):
    """A fit of noisy config-3 data with a validation set and
    early_stopping_rounds (E:2908-2935): the kept trees, best_iteration_,
    n_trees_fitted_, both loss histories and predict_proba."""
    X, y = D.config3(n=12_000)
    Xtr, ytr, Xva, yva, Xte = X[:6000], y[:6000], X[6000:9000], y[6000:9000], X[9000:]
    params = dict(n_estimators=80, max_depth=6, learning_rate=0.3, n_bins=128, class_weight="balanced_sqrt",
                  random_state=7, early_stopping_rounds=5)
    m = E.HybridHistGBMNumbaV1_0_1(verbose=False, **params)
    m.fit(Xtr, ytr, X_val=Xva, y_val=yva)
    T = len(m.trees)
    maxn = max(len(t[0]) for t in m.trees)
    arr = {k: np.full((T, maxn), fill, dtype=dt) for k, fill, dt in [
        ("tf", -1, np.int32), ("tt", 0, np.int64), ("tv", 0.0, np.float64),
        ("tl", -1, np.int32), ("tr", -1, np.int32), ("sg", 0.0, np.float64)]}
    ncs = np.zeros(T, dtype=np.int32)
    for t, (tf, tt, tv, tl, tr, nc, sg) in enumerate(m.trees):
        for k, a in zip(("tf", "tt", "tv", "tl", "tr", "sg"), (tf, tt, tv, tl, tr, sg)):
            arr[k][t, :len(a)] = a
        ncs[t] = nc
    np.savez_compressed(
        os.path.join(HERE, "fit_early.npz"), params=np.array(repr(params)), n_trees=T, nc=ncs, **arr,
        best_iteration=m.best_iteration_, n_trees_fitted=m.n_trees_fitted_, base_score=m.base_score_,
        learning_rate=m.learning_rate, max_leaves=m.max_leaves, max_depth=m.max_depth,
        min_child_weight=m.min_child_weight, subsample=m.subsample, colsample=m.colsample_bytree,
        reg_lambda=m.reg_lambda, gamma=m.gamma, min_samples_leaf=m.min_samples_leaf, n_bins=m.n_bins,
        binning_strategy=m.binning_strategy, edges=m.bin_edges, counts=m.feature_bin_counts,
        nan_bin_id=m._nan_bin_id, train_loss=np.array(m.train_loss_history_),
        val_loss=np.array(m.val_loss_history_), proba_test=m.predict_proba(Xte))
    return {"fit_early": (T, m.best_iteration_, len(m.val_loss_history_))}


def spw_case(E, D):
    """A fit of imbalanced config-2 data with objective='binary' and
    scale_pos_weight=3: the weighted bin edges (E:3211-3216, E:2073-2141)
    and the class weights (E:2572-2577) both use it."""
    X, y = D.config2(n=30_000, n_pos=150)
    Xtr, ytr, Xte = X[:24_000], y[:24_000], X[24_000:]
    params = dict(n_estimators=15, max_depth=5, n_bins=255, objective="binary", scale_pos_weight=3.0,
                  random_state=11)
    captured = []
    cls = E.HybridHistGBMNumbaV1_0_1
    orig = cls._build_one_tree

    def spy(self, X_bin, grad, hess, sample_idx, feat_idx, n_features):
        tree = orig(self, X_bin, grad, hess, sample_idx, feat_idx, n_features)
        captured.append((grad.copy(), hess.copy(), sample_idx.copy(), feat_idx.copy()))
        return tree

    cls._build_one_tree = spy
    try:
        m = cls(verbose=False, **params)
        m.fit(Xtr, ytr)
    finally:
        cls._build_one_tree = orig
    rounds = {}
    for r_, (g, h, smp, f) in enumerate(captured[:4]):
        rounds.update({f"r{r_}_g": g, f"r{r_}_h": h, f"r{r_}_sample": smp, f"r{r_}_feat": f})
    T = len(m.trees)
    maxn = max(len(t[0]) for t in m.trees)
    arr = {k: np.full((T, maxn), fill, dtype=dt) for k, fill, dt in [
        ("tf", -1, np.int32), ("tt", 0, np.int64), ("tv", 0.0, np.float64),
        ("tl", -1, np.int32), ("tr", -1, np.int32), ("sg", 0.0, np.float64)]}
    ncs = np.zeros(T, dtype=np.int32)
    for t, (tf, tt, tv, tl, tr, nc, sg) in enumerate(m.trees):
        for k, a in zip(("tf", "tt", "tv", "tl", "tr", "sg"), (tf, tt, tv, tl, tr, sg)):
            arr[k][t, :len(a)] = a
        ncs[t] = nc
    np.savez_compressed(
        os.path.join(HERE, "fit_spw.npz"), params=np.array(repr(params)), n_trees=T, nc=ncs, **arr, **rounds,
        base_score=m.base_score_, learning_rate=m.learning_rate, max_leaves=m.max_leaves,
        max_depth=m.max_depth, min_child_weight=m.min_child_weight, subsample=m.subsample,
        colsample=m.colsample_bytree, reg_lambda=m.reg_lambda, gamma=m.gamma,
        min_samples_leaf=m.min_samples_leaf, n_bins=m.n_bins, binning_strategy=m.binning_strategy,
        edges=m.bin_edges, counts=m.feature_bin_counts, nan_bin_id=m._nan_bin_id,
        train_loss=np.array(m.train_loss_history_), proba_test=m.predict_proba(Xte))
    return {"fit_spw": (T, float(m.base_score_))}


def main(ref_src, only=None):
    sys.path.insert(0, ref_src)
    import bsscl_gbm.estimator_v1_0_1 as E
    from bsscl_gbm_b200 import datasets as D

    out = {}
    if only in ("model", "multiclass", "regression", "monotone", "early", "spw"):
        if only == "model":
            out.update(model_json_case(E, D))
        elif only == "monotone":
            out.update(monotone_case(E, D))
        elif only == "early":
            out.update(early_stop_case(E, D))
        elif only == "spw":
            out.update(spw_case(E, D))
        elif only == "multiclass":
            out.update(multiclass_case(E, D))
        else:
            out.update(regression_case(E, D, "mse"))
            out.update(regression_case(E, D, "mae"))
        for k, v in out.items():
            print(k, v)
        return

    # ------------------------------------------------------------------
    # 1. Bin edges + binning (E:2073-2189, E:155-226)
    # ------------------------------------------------------------------
    def bin_case(name, X, n_bins, strategy):
        m = E.HybridHistGBMNumbaV1_0_1(n_bins=n_bins, verbose=False)
        m.categorical_features = None
        m.n_bins = n_bins
        edges, counts = m._build_bin_edges(X)
        m.bin_edges, m.feature_bin_counts = edges, counts
        m._max_bins = int(np.max(counts))
        m.binning_strategy = strategy
        Xb, _ = m._bin_features(X)
        np.savez_compressed(
            os.path.join(HERE, f"bin_{name}.npz"), X=X, n_bins=n_bins,
            strategy=strategy, edges=edges, counts=counts,
            nan_bin_id=m._nan_bin_id, X_bin=Xb.astype(np.uint16),
            dtype=str(Xb.dtype))
        out[f"bin_{name}"] = (Xb.dtype, int(Xb.max()), counts.max())

    rng = np.random.default_rng(100)
    X = rng.standard_normal((3000, 6))
    X[:, 1] = np.round(X[:, 1] * 2)            # few uniques
    X[:, 2] = 7.0                              # constant
    X[rng.random(3000) < 0.2, 3] = np.nan      # NaN column
    X[:, 4] = np.nan                           # all-NaN column
    X[:, 5] = rng.exponential(1.0, 3000) * 1e5  # large magnitudes
    for strat in ("standard", "hybrid"):
        bin_case(f"f64_{strat}", X, 255, strat)
        bin_case(f"f32_{strat}", X.astype(np.float32), 255, strat)
        bin_case(f"f64_nb32_{strat}", X, 32, strat)
    Xi = rng.integers(-20, 20, size=(2000, 4)).astype(np.float64)
    Xi[rng.random((2000, 4)) < 0.1] = np.nan
    bin_case("int_levels_hybrid", Xi, 255, "hybrid")
    bin_case("f32_nb254_standard", X.astype(np.float32), 254, "standard")

    # ------------------------------------------------------------------
    # 2. Direct tree-builder calls (E:517-823 leaf-wise, E:233-508 depth-wise)
    # ------------------------------------------------------------------
    def tree_case(name, n, p, nbins, seed, *, n_sub=None, n_feat=None,
                  max_leaves=63, max_depth=6, msl=5, mcw=1.0, lam=1.0,
                  gamma=0.0, gh="cont", clamp=False, const_feats=(),
                  nan_heavy=False, policy="leaf"):
        r = np.random.default_rng(seed)
        counts = np.full(p, nbins, dtype=np.int32)
        for j in const_feats:
            counts[j] = 1
        Xb = np.empty((n, p), dtype=np.uint16)
        for j in range(p):
            nb = counts[j]
            Xb[:, j] = r.integers(0, nb, n)
            if nan_heavy and nb > 2:
                Xb[r.random(n) < 0.3, j] = 0
            if clamp and nb > 2:
                Xb[r.random(n) < 0.02, j] = nb  # id one past the last bin
        if gh == "cont":
            g = r.standard_normal(n)
            h = r.uniform(0.01, 0.25, n)
        elif gh == "tied":
            yy = r.random(n) < 0.4
            g = np.where(yy, -0.6, 0.4)
            h = np.full(n, 0.24)
        elif gh == "weighted":
            yy = r.random(n) < 0.05
            w = np.where(yy, 7.27, 0.785)
            p_ = 1.0 / (1.0 + np.exp(-r.normal(-3, 1.0, n)))
            g = w * (p_ - yy)
            h = w * p_ * (1 - p_)
        n_sub = n if n_sub is None else n_sub
        n_feat = p if n_feat is None else n_feat
        sidx = r.permutation(n)[:n_sub].astype(np.int64)
        fidx = np.sort(r.permutation(p)[:n_feat]).astype(np.int32)
        max_bins = int(counts.max())
        is_cat = np.zeros(p, dtype=np.bool_)
        if policy == "leaf":
            t = E._build_tree_leafwise(
                Xb, g, h, sidx, fidx, np.int32(max_leaves), np.int32(max_depth),
                np.int32(msl), np.float64(mcw), counts, np.int32(max_bins),
                np.float64(lam), np.float64(gamma), np.int32(p), is_cat)
        else:
            t = E._build_tree_v25(
                Xb, g, h, sidx, fidx, np.int32(max_depth), np.int32(msl),
                np.float64(mcw), counts, np.int32(max_bins), np.float64(lam),
                np.float64(gamma), np.int32(p), is_cat)
        tf, tt, tv, tl, tr, nc, sg = [np.array(a) for a in t]
        tfp, tlp, trp = tf.copy(), tl.copy(), tr.copy()
        E._post_prune_tree_jit(tfp, tlp, trp, sg, np.float64(gamma), int(nc))
        leaf = E.predict_batch_jit(Xb, tfp[:nc], tt[:nc], np.arange(nc, dtype=np.float64),
                                   tlp[:nc], trp[:nc], np.zeros(p, dtype=np.bool_))
        np.savez_compressed(
            os.path.join(HERE, f"tree_{name}.npz"), X_bin=Xb, g=g, h=h,
            sample_idx=sidx, feat_idx=fidx, counts=counts, max_leaves=max_leaves,
            max_depth=max_depth, msl=msl, mcw=mcw, lam=lam, gamma=gamma,
            policy=policy, tf=tf, tt=tt, tv=tv, tl=tl, tr=tr, nc=nc, sg=sg,
            tf_pruned=tfp, tl_pruned=tlp, tr_pruned=trp,
            leaf_of_row=leaf.astype(np.int32))
        out[f"tree_{name}"] = int(nc)

    tree_case("basic", 6000, 16, 256, 1)
    tree_case("subsample", 8000, 24, 256, 2, n_sub=6000, n_feat=17)
    tree_case("gamma", 5000, 12, 64, 3, gamma=0.8)
    tree_case("msl_big", 4000, 10, 256, 4, msl=300)
    tree_case("mcw_big", 4000, 10, 256, 5, mcw=60.0)
    tree_case("depth3", 5000, 12, 256, 6, max_depth=3)
    tree_case("leaves4", 5000, 12, 256, 7, max_leaves=4)
    tree_case("const_clamp", 5000, 12, 100, 8, const_feats=(0, 5), clamp=True)
    tree_case("nan_heavy", 6000, 14, 256, 9, nan_heavy=True, gh="weighted",
              mcw=3.0, lam=1.0)
    tree_case("tiny", 3, 4, 8, 10)
    tree_case("tied", 3000, 10, 32, 11, gh="tied", max_leaves=31)
    tree_case("lam5", 5000, 12, 256, 12, lam=5.0, mcw=3.0)
    tree_case("few_bins", 5000, 20, 2, 13)
    tree_case("level_basic", 5000, 12, 256, 14, policy="level", max_depth=5)
    tree_case("level_gamma", 5000, 12, 64, 15, policy="level", max_depth=4,
              gamma=0.5, msl=50)

    # ------------------------------------------------------------------
    # 3. NumPy legacy RandomState shuffle stream (E:2502-2517)
    # ------------------------------------------------------------------
    seqs = {}
    for seed, n, p, frac, fc, rounds in [(0, 1000, 30, 0.8, 0.8, 5),
                                         (7, 70000, 100, 0.75, 0.7, 3),
                                         (4294967295, 17, 3, 0.5, 0.5, 4)]:
        rs = np.random.RandomState(seed)
        allr = np.arange(n, dtype=np.int64)
        allf = np.arange(p, dtype=np.int32)
        ns, nf = max(1, int(n * frac)), max(1, int(p * fc))
        for r_ in range(rounds):
            rs.shuffle(allr)
            s = allr[:ns].copy()
            rs.shuffle(allf)
            f = np.sort(allf[:nf]).copy()
            seqs[f"s{seed}_n{n}_r{r_}_sample"] = s
            seqs[f"s{seed}_n{n}_r{r_}_feat"] = f
    np.savez_compressed(os.path.join(HERE, "sampler.npz"), **seqs)

    # ------------------------------------------------------------------
    # 4. Ensemble predict (E:863-884) on a random packed ensemble
    # ------------------------------------------------------------------
    ens = D.config5_ensemble(n_trees=40, depth=5, p=12, seed=21, max_threshold=60)
    rng = np.random.default_rng(22)
    Xb = rng.integers(0, 64, size=(3000, 12)).astype(np.uint16)
    F = E.predict_all_trees_jit(
        Xb, ens["features"], ens["thresholds"], ens["values"], ens["left"],
        ens["right"], ens["offsets"], np.int32(40), np.float64(0.08),
        np.zeros(12, dtype=np.bool_))
    np.savez_compressed(os.path.join(HERE, "predict_ensemble.npz"), X_bin=Xb, F=F,
                        lr=0.08, **ens)

    # ------------------------------------------------------------------
    # 5. Full binary fits with per-round capture
    # ------------------------------------------------------------------
    def fit_case(name, X, y, X_test, params, keep_rounds=4):
        captured = []
        cls = E.HybridHistGBMNumbaV1_0_1
        orig = cls._build_one_tree

        def spy(self, X_bin, grad, hess, sample_idx, feat_idx, n_features):
            tree = orig(self, X_bin, grad, hess, sample_idx, feat_idx, n_features)
            captured.append((grad.copy(), hess.copy(), sample_idx.copy(), feat_idx.copy()))
            return tree

        cls._build_one_tree = spy
        try:
            m = cls(verbose=False, **params)
            m.fit(X, y)
        finally:
            cls._build_one_tree = orig
        Xb_train, _ = m._bin_features(X if np.issubdtype(X.dtype, np.floating) else X.astype(np.float64))
        proba_test = m.predict_proba(X_test)
        proba_train = m.predict_proba(X)
        T = len(m.trees)
        maxn = max(len(t[0]) for t in m.trees)
        arr = {k: np.full((T, maxn), fill, dtype=dt) for k, fill, dt in [
            ("tf", -1, np.int32), ("tt", 0, np.int64), ("tv", 0.0, np.float64),
            ("tl", -1, np.int32), ("tr", -1, np.int32), ("sg", 0.0, np.float64)]}
        ncs = np.zeros(T, dtype=np.int32)
        for t, (tf, tt, tv, tl, tr, nc, sg) in enumerate(m.trees):
            for k, a in zip(("tf", "tt", "tv", "tl", "tr", "sg"), (tf, tt, tv, tl, tr, sg)):
                arr[k][t, :len(a)] = a
            ncs[t] = nc
        extra = {}
        for r_ in range(min(keep_rounds, T)):
            g, h, s, f = captured[r_]
            extra[f"r{r_}_g"] = g
            extra[f"r{r_}_h"] = h
            extra[f"r{r_}_sample"] = s
            extra[f"r{r_}_feat"] = f
        sample_sha = np.array([sha(c[2]) for c in captured])
        feat_sha = np.array([sha(c[3]) for c in captured])
        np.savez_compressed(
            os.path.join(HERE, f"fit_{name}.npz"),
            params=np.array(repr(params)), n_trees=T, nc=ncs, **arr, **extra,
            base_score=m.base_score_, learning_rate=m.learning_rate,
            max_leaves=m.max_leaves, max_depth=m.max_depth,
            min_child_weight=m.min_child_weight, subsample=m.subsample,
            colsample=m.colsample_bytree, reg_lambda=m.reg_lambda,
            gamma=m.gamma, min_samples_leaf=m.min_samples_leaf,
            binning_strategy=m.binning_strategy, n_bins=m.n_bins,
            edges=m.bin_edges, counts=m.feature_bin_counts,
            nan_bin_id=m._nan_bin_id, max_bins=m._max_bins,
            X_bin_sha=sha(Xb_train.astype(np.uint16)),
            X_bin=Xb_train.astype(np.uint16) if Xb_train.size <= 600_000 else np.zeros(0),
            train_loss=np.array(m.train_loss_history_),
            proba_test=proba_test, proba_train=proba_train,
            sample_sha=sample_sha, feat_sha=feat_sha,
            packed_features=m._packed_features, packed_thresholds=m._packed_thresholds,
            packed_values=m._packed_values, packed_left=m._packed_left,
            packed_right=m._packed_right, tree_offsets=m._tree_offsets,
            feature_importances=m.feature_importances_,
            class_weight=np.array(str(params.get("class_weight", "balanced_sqrt"))))
        out[f"fit_{name}"] = (T, float(proba_test[:, 1].mean()))

    Xtr, ytr, Xte, yte = D.config1()
    fit_case("cfg1", Xtr, ytr, Xte, dict(n_estimators=100, max_depth=6, learning_rate=0.1,
                                          n_bins=255, class_weight=None, random_state=0))
    X2, y2 = D.config2(n=40_000, n_pos=120)
    fit_case("cfg2_small", X2[:32_000], y2[:32_000], X2[32_000:],
             dict(n_estimators=30, max_depth=6, class_weight="balanced_sqrt",
                  n_bins=255, random_state=0))
    X3, y3 = D.config3(n=25_000)
    fit_case("cfg3_small", X3[:20_000], y3[:20_000], X3[20_000:],
             dict(n_estimators=30, max_depth=6, class_weight="balanced_sqrt",
                  n_bins=255, random_state=0))
    X4, y4 = D.config4(n=30_000)
    fit_case("cfg4_small", X4[:24_000], y4[:24_000], X4[24_000:],
             dict(n_estimators=10, max_depth=8, n_bins=255, random_state=0))
    fit_case("cfg1_level", Xtr[:4000], ytr[:4000], Xte,
             dict(n_estimators=20, max_depth=4, learning_rate=0.1, n_bins=64,
                  class_weight="balanced", random_state=3, grow_policy="level"))
    out.update(model_json_case(E, D))
    out.update(multiclass_case(E, D))
    out.update(regression_case(E, D, "mse"))
    out.update(regression_case(E, D, "mae"))
    out.update(monotone_case(E, D))
    out.update(early_stop_case(E, D))
    out.update(spw_case(E, D))

    for k, v in out.items():
        print(k, v)


if __name__ == "__main__":
    # python make_golden.py <reference>/src [model]   ('model': only the save_model fixture)
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference>/src [model|multiclass|regression|monotone|early|spw]")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else None)
