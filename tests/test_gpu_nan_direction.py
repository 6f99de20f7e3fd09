"""The learned NaN direction (gbm_params.nan_direction, the estimator's
nan_direction='learn'; no reference counterpart -- the reference always sends
the NaN bin left, E:668) on the GPU, against the oracle's restatement of the
two-direction scan (oracle.c find_split with nan_bin_id):

* round after round, the engine's tree (features, thresholds, NaN
  directions, children, values, gains), per-row leaf ids and F update equal
  the oracle's EXACT tree on the engine's own gradients, best-first and
  depth-wise;
* an estimator fit with nan_direction='learn' learns NaN-right splits, and
  its predict_proba equals the oracle's walk of its packed ensemble, before
  and after a JSON round trip;
* the predict kernel honours NaN-right splits in both node formats.

With the flag off every parity test of the reference's NaN-left rule holds
unchanged (tests/test_gpu_parity.py, tests/test_gpu_full_parity.py).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _nan_data(n=20_000, p=12, seed=5):
    """NaN in four features; in two of them the NaN rows' labels follow the
    high values, so sending NaN right gains more there."""
    from bsscl_gbm_b200 import binning
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, p))
    logit = 1.5 * (X[:, 0] > 0.7) + 1.2 * (X[:, 1] > 0.5) + 0.5 * X[:, 2] - 1.0
    y = (rng.random(n) < 1.0 / (1.0 + np.exp(-logit))).astype(np.int64)
    for j, frac in ((0, 0.3), (1, 0.25), (5, 0.2), (7, 0.1)):
        m = rng.random(n) < frac
        if j in (0, 1):
            y[m] = (rng.random(m.sum()) < 0.85).astype(np.int64)
        X[m, j] = np.nan
    e, c, nb = binning.build_bin_edges(X, 128)
    Xb = binning.bin_features(X, e, c, nb)
    return X, y, Xb, e, c, nb


def _params(nb, policy="leaf", lr=0.1):
    from bsscl_gbm_b200 import GbmParams
    from bsscl_gbm_b200._lib import with_nan_direction
    prm = GbmParams(1.0, 0.0, 1.0, lr, 5, 6 if policy == "leaf" else 4, 31, 0 if policy == "leaf" else 1, None)
    return with_nan_direction(prm, nb)


@pytest.mark.parametrize("policy", ["leaf", "level"])
def test_rounds_match_oracle_with_nan_direction(engine, policy):
    from bsscl_gbm_b200 import Sampler, binning
    X, y, Xb, e, counts, nanb = _nan_data()
    n, p = Xb.shape
    w2 = O.class_weights(y, None)
    base = O.base_score(y, w2)
    engine.upload_bins(binning.device_bins(Xb, counts), counts)
    engine.upload_labels(y.astype(np.uint8), w2, base, n_global=n)
    prm, keep = _params(nanb, policy)
    cap = 64 if policy == "leaf" else 31
    S = engine.scale_bits()
    s = Sampler(3, n, p, int(n * 0.8), int(p * 0.75), True, True)
    F_prev = engine.get_F()
    y8 = y.astype(np.uint8)
    n_right = 0
    for r in range(5):
        g, h = engine.get_grad()
        smp, mask, feat = s.next(want_sample=True, want_mask=True)
        tree, loss, leaf = engine.round(mask, feat, prm, cap, want_leaf=True)
        assert len(tree) == 8
        kw = dict(max_leaves=31, max_depth=6, msl=5, mcw=1.0, lam=1.0) if policy == "leaf" else \
            dict(max_depth=4, msl=5, mcw=1.0, lam=1.0)
        o = O.build_tree(Xb, g, h, smp, feat, counts, mode=O.MODE_EXACT, scale_bits=S, policy=policy,
                         nan_bin_id=nanb, **kw)
        O.post_prune(o[0], o[3], o[4], o[6], 0.0, o[5])
        othr, onr = O.split_nan_right(o[1])
        nc = tree[5]
        assert nc == o[5], f"round {r}: {nc} vs {o[5]} nodes"
        for a, b, what in ((tree[0], o[0], "features"), (tree[1], othr, "thresholds"), (tree[7], onr, "NaN"),
                           (tree[3], o[3], "left"), (tree[4], o[4], "right"), (tree[2], o[2], "values"),
                           (tree[6], o[6], "gains")):
            assert np.array_equal(np.asarray(a)[:nc], np.asarray(b)[:nc]), f"round {r}: {what}"
        n_right += int(np.sum(np.asarray(tree[7])[:nc][np.asarray(tree[0])[:nc] >= 0]))
        assert np.array_equal(leaf, O.leaf_ids(Xb, tree[0][:nc], tree[1][:nc], tree[3][:nc], tree[4][:nc],
                                               nan_right=tree[7][:nc]))
        F = engine.get_F()
        assert np.array_equal(F, F_prev + 0.1 * tree[2][leaf])
        assert abs(loss - O.logloss(F, y8)) <= 1e-12 * max(1.0, abs(loss))
        F_prev = F
    s.close()
    assert n_right > 0, "no split learned to send NaN right"


def test_estimator_learns_nan_direction_and_predicts_with_it(tmp_path):
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M, binning
    X, y, _, _, _, _ = _nan_data(n=30_000, seed=8)
    Xtr, ytr, Xte = X[:24_000], y[:24_000], X[24_000:]
    m = M(n_estimators=25, max_depth=5, learning_rate=0.1, n_bins=128, class_weight=None, random_state=0,
          nan_direction='learn', verbose=False).fit(Xtr, ytr)
    m_left = M(n_estimators=25, max_depth=5, learning_rate=0.1, n_bins=128, class_weight=None, random_state=0,
               verbose=False).fit(Xtr, ytr)
    assert m._packed_nan_right is not None and m._packed_nan_right.sum() > 0
    assert m_left._packed_nan_right is None
    Xb = binning.bin_features(Xte, m.bin_edges, m.feature_bin_counts, m._nan_bin_id)
    F = O.predict_packed(Xb, m._packed(), len(m.trees), m.learning_rate) + m.base_score_
    P = m.predict_proba(Xte)[:, 1]
    assert np.abs(P - 1.0 / (1.0 + np.exp(-F))).max() <= 1e-12
    # the learned direction fits the training rows at least as well here
    assert m.train_loss_history_[-1] <= m_left.train_loss_history_[-1]
    path = str(tmp_path / "m.json")
    m.save_model(path)
    back = M.load_model(path)
    assert np.array_equal(back._packed_nan_right, m._packed_nan_right)
    assert np.abs(back.predict_proba(Xte) - m.predict_proba(Xte)).max() == 0.0


@pytest.mark.parametrize("p", [40, 3000])
def test_predict_honours_nan_right_in_both_node_formats(engine, p):
    """p = 40: 32-bit breadth-first nodes (NaN-right threshold stored as t -
    1, bin - 1 mod 256 compared); p = 3000: 8-byte nodes."""
    from bsscl_gbm_b200 import datasets as D
    rng = np.random.default_rng(p)
    n = 4000 if p < 1000 else 600
    Xb = rng.integers(0, 256, size=(n, p)).astype(np.uint8)
    Xb[rng.random((n, p)) < 0.2] = 0                      # plenty of NaN-bin entries
    ens = D.config5_ensemble(n_trees=20, depth=7, p=p, seed=p, max_threshold=253)
    internal = ens["features"] >= 0
    nr = (internal & (rng.random(len(internal)) < 0.5) & (ens["thresholds"] >= 1)).astype(np.uint8)
    ens["nan_right"] = nr
    F, P = engine.predict(Xb, ens, 20, 0.08, 0.3)
    Fo = O.predict_packed(Xb, ens, 20, 0.08) + 0.3
    assert np.abs(F - Fo).max() <= 1e-12
    bad = dict(ens)
    bad["nan_right"] = nr.copy()
    bad["thresholds"] = ens["thresholds"].copy()
    k = int(np.flatnonzero(nr)[0])
    bad["thresholds"][k] = 0                              # a NaN-right split needs threshold >= 1
    with pytest.raises(RuntimeError, match="NaN-right split needs threshold"):
        engine.predict(Xb, bad, 20, 0.08, 0.3)
