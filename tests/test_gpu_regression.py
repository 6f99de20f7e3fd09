"""Regression on the GPU (gbm_upload_targets / gbm_round_reg), through the
C ABI, on a B200.

* Round after round, the tree == the oracle's EXACT builder on the engine's
  own quantised gradients and fixed-point exponent (which follows the
  round's largest |g|), bit for bit; F moves by exactly lr * value(leaf).
* The regressor's fit vs the reference's recorded fits (mse and mae):
  identical trees until a divergence, which must be an exact tie of the
  reference's own round inputs; predictions within 1e-6 (relative).
* A fitted regressor survives save_model / load_model.
"""
import ast

import numpy as np
import pytest

import audit as A
import oracle as O
from helpers import fit_inputs, golden, golden_trees, reg_fit_kwargs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("loss", ["mse", "mae"])
def test_reg_rounds_match_oracle_exact(engine, loss):
    from bsscl_gbm_b200 import GbmParams
    d = golden(f"fit_reg_{loss}")
    X, y, _ = fit_inputs("reg")
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    kw = reg_fit_kwargs(d)
    prm = GbmParams(kw["reg_lambda"], kw["gamma"], kw["min_child_weight"], kw["learning_rate"],
                    kw["min_samples_leaf"], kw["max_depth"], kw["max_leaves"], 0, None)
    cap = 2 * kw["max_leaves"] + 2
    n, p = Xb.shape
    engine.upload_bins(Xb, d["counts"])
    engine.upload_targets(y, float(np.mean(y)), loss)
    rng = np.random.default_rng(8)
    for r in range(4):
        g, h = engine.get_grad()
        S = engine.scale_bits()
        F0 = engine.get_F()
        want_g = F0 - y if loss == "mse" else np.sign(F0 - y)
        assert S == O.reg_scale_bits(1.0 if loss == "mae" else np.max(np.abs(want_g)))
        assert np.array_equal(g, np.rint(np.ldexp(want_g, S)) / 2.0 ** S)
        mask = (rng.random(n) < 0.75).astype(np.uint8)
        smp = np.nonzero(mask)[0].astype(np.int64)
        feat = np.sort(rng.choice(p, size=7, replace=False)).astype(np.int32)
        tree, tloss, leaf = engine.round_reg(mask, feat, prm, cap, want_leaf=True)
        o = O.build_tree(Xb, g, h, smp, feat, d["counts"], max_leaves=kw["max_leaves"], max_depth=kw["max_depth"],
                         msl=kw["min_samples_leaf"], mcw=kw["min_child_weight"], lam=kw["reg_lambda"],
                         gamma=kw["gamma"], mode=O.MODE_EXACT, scale_bits=S)
        O.post_prune(o[0], o[3], o[4], o[6], kw["gamma"], o[5])
        nc = tree[5]
        assert nc == o[5], f"round {r}: {nc} vs {o[5]} nodes"
        for i in (0, 1, 2, 3, 4, 6):
            assert np.array_equal(np.asarray(tree[i])[:nc], np.asarray(o[i])[:nc]), f"round {r} field {i}"
        F1 = engine.get_F()
        assert np.array_equal(F1, F0 + kw["learning_rate"] * tree[2][leaf])
        want = np.mean((y - F1) ** 2) if loss == "mse" else np.mean(np.abs(y - F1))
        assert abs(tloss - want) <= 1e-12 * max(1.0, abs(want))


@pytest.mark.parametrize("loss", ["mse", "mae"])
def test_regressor_fit_matches_reference(loss):
    from bsscl_gbm_b200 import HybridHistGBMRegressorV1_0_1 as R
    d = golden(f"fit_reg_{loss}")
    X, y, Xte = fit_inputs("reg")
    m = R(verbose=False, **ast.literal_eval(str(d["params"]))).fit(X, y)
    assert m.init_score_ == float(d["init_score"])
    ref = golden_trees(d)
    assert len(m.trees) == len(ref)
    div = A.first_divergence(ref, m.trees)
    upto = len(ref) if div is None else div[0]
    for t in range(upto):
        nc = ref[t][5]
        scale = max(1.0, np.abs(ref[t][2][:nc]).max())
        assert np.abs(m.trees[t][2][:nc] - ref[t][2][:nc]).max() <= 1e-6 * scale, f"values tree {t}"
    if div is None:
        pred = m.predict(Xte)
        assert np.abs(pred - d["pred_test"]).max() <= 1e-6 * max(1.0, np.abs(d["pred_test"]).max())
        assert np.abs(np.array(m.train_loss_history_) - d["train_loss"]).max() <= 1e-9 * d["train_loss"].max()
        return
    t = div[0]
    assert f"r{t}_g" in d.files, f"divergence at tree {t} beyond the recorded rounds"
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    res = A.audit_node(Xb, d[f"r{t}_g"], d[f"r{t}_h"], d[f"r{t}_sample"], d["counts"], ref[t], m.trees[t], div[1],
                       float(d["reg_lambda"]), float(d["min_child_weight"]))
    assert A.explained(res), res


def test_regressor_model_json_round_trip(tmp_path):
    from bsscl_gbm_b200 import HybridHistGBMRegressorV1_0_1 as R
    X, y, Xte = fit_inputs("reg")
    m = R(n_estimators=5, max_depth=4, n_bins=64, random_state=2, verbose=False).fit(X, y)
    path = str(tmp_path / "reg.json")
    m.save_model(path)
    b = R.load_model(path)
    assert b.init_score_ == m.init_score_
    assert np.array_equal(b.predict(Xte), m.predict(Xte))
