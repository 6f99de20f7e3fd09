"""Multi-class softmax on the GPU (gbm_upload_labels_mc / gbm_round_mc),
through the C ABI, on a B200.

* Round after round, every class's tree == the oracle's EXACT builder on the
  engine's own quantised gradients of that class, bit for bit, and F of each
  class moves by exactly lr * value(leaf).
* The estimator's multi-class fit vs the reference's recorded fit
  (tests/golden/fit_mc.npz): identical trees until a divergence, which must be
  an exact tie of the reference's own round inputs; predict_proba within 1e-6.
* A fitted multi-class model survives save_model / load_model.
"""
import numpy as np
import pytest

import audit as A
import oracle as O
from helpers import fit_inputs, golden, golden_mc_trees, mc_fit_kwargs, same_topology

pytestmark = pytest.mark.gpu


def _params(d):
    from bsscl_gbm_b200 import GbmParams
    kw = mc_fit_kwargs(d)
    return GbmParams(kw["reg_lambda"], kw["gamma"], kw["min_child_weight"], kw["learning_rate"],
                     kw["min_samples_leaf"], kw["max_depth"], kw["max_leaves"], 0, None), kw


def test_mc_rounds_match_oracle_exact(engine):
    d = golden("fit_mc")
    X, y, _ = fit_inputs("mc")
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    K = int(d["n_classes"])
    n, p = Xb.shape
    prm, kw = _params(d)
    cap = 2 * kw["max_leaves"] + 2
    engine.upload_bins(Xb, d["counts"])
    w = O.class_weights_mc(y, K, "balanced_sqrt")
    engine.upload_labels_mc(y.astype(np.uint8), K, w)
    S = engine.scale_bits()
    rng = np.random.default_rng(5)
    lr = kw["learning_rate"]
    for r in range(4):
        mask = (rng.random(n) < 0.8).astype(np.uint8)
        smp = np.nonzero(mask)[0].astype(np.int64)
        feat = np.sort(rng.choice(p, size=9, replace=False)).astype(np.int32)
        gh = [engine.get_grad_mc(k) for k in range(K)]
        F0 = engine.get_F_mc()
        trees, loss, leaves = engine.round_mc(mask, feat, prm, cap, want_leaf=True)
        F1 = engine.get_F_mc()
        for k in range(K):
            o = O.build_tree(Xb, gh[k][0], gh[k][1], smp, feat, d["counts"], max_leaves=kw["max_leaves"],
                             max_depth=kw["max_depth"], msl=kw["min_samples_leaf"], mcw=kw["min_child_weight"],
                             lam=kw["reg_lambda"], gamma=kw["gamma"], mode=O.MODE_EXACT, scale_bits=S)
            O.post_prune(o[0], o[3], o[4], o[6], kw["gamma"], o[5])
            t = trees[k]
            nc = t[5]
            assert nc == o[5], f"round {r} class {k}: {nc} vs {o[5]} nodes"
            for i in (0, 1, 2, 3, 4, 6):
                assert np.array_equal(np.asarray(t[i])[:nc], np.asarray(o[i])[:nc]), f"round {r} class {k} field {i}"
            assert np.array_equal(F1[k], F0[k] + lr * t[2][leaves[k]]), f"round {r} class {k} F"
        Fr = F1.T
        want = O.mc_logloss(np.eye(K)[y], Fr)
        assert abs(loss - want) <= 1e-12 * max(1.0, abs(want))


def test_mc_fit_matches_reference():
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    import ast
    d = golden("fit_mc")
    X, y, Xte = fit_inputs("mc")
    params = ast.literal_eval(str(d["params"]))
    m = M(verbose=False, **params).fit(X, y)
    assert m._is_multiclass and m.n_classes_ == int(d["n_classes"])
    ref = golden_mc_trees(d)
    K, T = int(d["n_classes"]), int(d["n_trees"])
    # the reference builds class 0..K-1 of round 0, then of round 1, ...
    mine = [m.mc_trees[k][t] for t in range(T) for k in range(K)]
    theirs = [ref[k][t] for t in range(T) for k in range(K)]
    div = A.first_divergence(theirs, mine)
    upto = len(theirs) if div is None else div[0]
    for j in range(upto):
        nc = theirs[j][5]
        assert np.abs(mine[j][2][:nc] - theirs[j][2][:nc]).max() <= 1e-6, f"values of tree {j}"
    if div is None:
        assert np.abs(m.predict_proba(Xte) - d["proba_test"]).max() <= 1e-6
        assert np.abs(np.array(m.train_loss_history_) - d["train_loss"]).max() <= 1e-9
        assert np.array_equal(m.predict(Xte), m.classes_[np.argmax(d["proba_test"], axis=1)])
        return
    j = div[0]
    t, k = divmod(j, K)
    assert f"r{t}_k{k}_g" in d.files, f"divergence at round {t} beyond the recorded rounds"
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    res = A.audit_node(Xb, d[f"r{t}_k{k}_g"], d[f"r{t}_k{k}_h"], d[f"r{t}_sample"], d["counts"], theirs[j],
                       mine[j], div[1], float(d["reg_lambda"]), float(d["min_child_weight"]))
    assert A.explained(res), res


def test_mc_model_json_round_trip(tmp_path):
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    X, y, Xte = fit_inputs("mc")
    m = M(n_estimators=4, max_depth=4, n_bins=64, random_state=3, verbose=False).fit(X, y)
    path = str(tmp_path / "mc.json")
    m.save_model(path)
    b = M.load_model(path)
    assert b._is_multiclass and len(b.mc_trees) == m.n_classes_
    assert np.array_equal(b.predict_proba(Xte), m.predict_proba(Xte))
    assert np.array_equal(b.predict(Xte), m.predict(Xte))
