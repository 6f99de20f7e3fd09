"""Features with 257 bin ids on the GPU.

The reference's default ``n_bins='auto'`` is 256 once p >= 28 (E:223-224
of the estimator's fit), and _build_bin_edges then gives every continuous
feature 257 bins (ids 0..256, E:2111-2127): the uint16 bin matrix of
_bin_features.  The engine keeps min(id, 255) in its byte matrix and the
rows of id 256 as a bit per row; the split search subtracts their top cell
from bin 255 at threshold 255, and the partition, the F update and the
predict walk send a row of bin 256 right at threshold 255.

* Round after round, from the reference's uint16 ids (gbm_upload_bins_u16),
  the engine's trees, leaf ids and F equal the oracle's EXACT trees on the
  engine's own gradients, best-first and depth-wise, with splits at
  threshold 255 among them.
* A model with splits at threshold 255 predicts the oracle's walk of the
  uint16 ids through every predict entry: raw rows binned on the GPU
  (gbm_predict_raw), uint16 ids (gbm_predict_upload_u16), and a threshold
  above 255 (every bin left).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _bins(n=20_000, seed=21):
    from bsscl_gbm_b200 import binning, datasets as D
    X, y = D.top_bin(n=n, seed=seed)
    e, c, nb = binning.build_bin_edges(X, 256)
    Xb = binning.bin_features(X, e, c, nb)
    return X, y, Xb, e, c, nb


@pytest.mark.parametrize("policy", ["leaf", "level"])
def test_rounds_from_uint16_ids_match_oracle(engine, policy):
    from bsscl_gbm_b200 import GbmParams, Sampler
    X, y, Xb, e, counts, nanb = _bins()
    assert Xb.dtype == np.uint16 and int(np.max(counts)) == 257 and int(Xb.max()) == 256
    n, p = Xb.shape
    w2 = O.class_weights(y, "balanced_sqrt")
    base = O.base_score(y, w2)
    engine.upload_bins(Xb, counts)
    engine.upload_labels(y.astype(np.uint8), w2, base, n_global=n)
    prm = GbmParams(1.0, 0.0, 1.0, 0.2, 5, 6 if policy == "leaf" else 5, 63, 0 if policy == "leaf" else 1, None)
    cap = 2 * 63 + 2 if policy == "leaf" else 63
    S = engine.scale_bits()
    s = Sampler(0, n, p, int(n * 0.8), int(p * 0.8), True, True)
    F_prev = engine.get_F()
    y8 = y.astype(np.uint8)
    n255 = 0
    for r in range(12):
        g, h = engine.get_grad()
        smp, mask, feat = s.next(want_sample=True, want_mask=True)
        tree, loss, leaf = engine.round(mask, feat, prm, cap, want_leaf=True)
        kw = dict(max_leaves=63, max_depth=6, msl=5, mcw=1.0, lam=1.0) if policy == "leaf" else \
            dict(max_depth=5, msl=5, mcw=1.0, lam=1.0)
        o = O.build_tree(Xb, g, h, smp, feat, counts, mode=O.MODE_EXACT, scale_bits=S, policy=policy, **kw)
        O.post_prune(o[0], o[3], o[4], o[6], 0.0, o[5])
        nc = tree[5]
        assert nc == o[5], f"round {r}: {nc} vs {o[5]} nodes"
        for a, b, what in ((tree[0], o[0], "features"), (tree[1], o[1], "thresholds"), (tree[3], o[3], "left"),
                           (tree[4], o[4], "right"), (tree[2], o[2], "values"), (tree[6], o[6], "gains")):
            assert np.array_equal(np.asarray(a)[:nc], np.asarray(b)[:nc]), f"round {r}: {what}"
        internal = np.asarray(tree[0])[:nc] >= 0
        n255 += int(np.sum(internal & (np.asarray(tree[1])[:nc] == 255)))
        assert np.array_equal(leaf, O.leaf_ids(Xb, tree[0][:nc], tree[1][:nc], tree[3][:nc], tree[4][:nc]))
        F = engine.get_F()
        assert np.array_equal(F, F_prev + 0.2 * tree[2][leaf])
        assert abs(loss - O.logloss(F, y8)) <= 1e-12 * max(1.0, abs(loss))
        F_prev = F
    s.close()
    assert n255 > 0, "no split at threshold 255"


def test_predict_entries_send_bin_256_right_at_threshold_255(engine):
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M, binning
    X, y, _, _, _, _ = _bins()
    Xh, _ = __import__("bsscl_gbm_b200.datasets", fromlist=["top_bin"]).top_bin(n=5_000, seed=22)
    m = M(n_estimators=20, random_state=0, verbose=False).fit(X, y)
    assert int(np.max(m.feature_bin_counts)) == 257
    pk = m._packed()
    internal = pk["features"] >= 0
    assert np.sum(internal & (pk["thresholds"] == 255)) > 0
    Xb = binning.bin_features(Xh, m.bin_edges, m.feature_bin_counts, m._nan_bin_id)
    assert Xb.dtype == np.uint16 and int(Xb.max()) == 256
    Fo = O.predict_packed(Xb, pk, len(m.trees), m.learning_rate) + m.base_score_
    Po = 1.0 / (1.0 + np.exp(-Fo))
    # raw rows binned on the GPU
    assert np.abs(m.predict_proba(Xh)[:, 1] - Po).max() <= 1e-12
    # the reference's uint16 ids
    assert np.abs(m.predict_proba_binned(Xb)[:, 1] - Po).max() <= 1e-12
    F, _ = engine.predict(Xb, pk, len(m.trees), m.learning_rate, m.base_score_, want_proba=False)
    assert np.abs(F - Fo).max() <= 1e-12
    # a threshold above 255 sends every bin left, 256 included
    big = dict(pk)
    big["thresholds"] = pk["thresholds"].copy()
    k = np.flatnonzero(internal & (pk["thresholds"] == 255))
    big["thresholds"][k] = 300
    F2, _ = engine.predict(Xb, big, len(m.trees), m.learning_rate, m.base_score_, want_proba=False)
    assert np.abs(F2 - (O.predict_packed(Xb, big, len(m.trees), m.learning_rate) + m.base_score_)).max() <= 1e-12
    assert np.abs(F2 - F).max() > 0.0
