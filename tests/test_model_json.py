"""Model JSON (save_model / load_model, E:4035-4205).

* A file written by the reference's own save_model loads with the
  reference's semantics (every feature NaN-free, trees and edges as saved).
* save_model writes every key the reference writes, plus the NaN bins and
  the resolved hyper-parameters; a save -> load round trip keeps all of them.
* On a GPU: the loaded reference model predicts what the reference predicts
  after its own reload, and a fitted model with NaN features predicts the
  same before and after a round trip.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from helpers import fit_inputs

REF_JSON = os.path.join(GOLDEN, "model_ref_cfg3.json")


def _model_cls():
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1
    return HybridHistGBMNumbaV1_0_1


def test_loads_reference_json():
    with open(REF_JSON) as f:
        data = json.load(f)
    m = _model_cls().load_model(REF_JSON)
    assert len(m.trees) == len(data["trees"]) == m.n_trees_fitted_
    assert np.array_equal(m.bin_edges, np.array(data["bin_edges"]))
    assert np.array_equal(m.feature_bin_counts, np.array(data["feature_bin_counts"]))
    assert np.all(m._nan_bin_id == -1)                  # the reference's reload rule
    assert m.learning_rate == data["params"]["learning_rate"]
    assert m.base_score_ == data["base_score_"]
    for t, td in zip(m.trees, data["trees"]):
        nc = td["node_count"]
        assert t[5] == nc
        assert np.array_equal(t[0][:nc], td["features"][:nc])
        assert np.array_equal(t[1][:nc], td["thresholds"][:nc])
        assert np.array_equal(t[2][:nc], td["values"][:nc])
    assert m._tree_offsets[-1] == sum(td["node_count"] for td in data["trees"])


def test_save_writes_reference_keys_and_round_trips(tmp_path):
    with open(REF_JSON) as f:
        ref_keys = set(json.load(f))
    M = _model_cls()
    m = M.load_model(REF_JSON)
    m._nan_bin_id = np.where(np.arange(m.n_features_in_) % 3 == 0, 0, -1).astype(np.int32)
    m.learning_rate = 0.0625                            # a resolved value the params do not show
    path = str(tmp_path / "m.json")
    m.save_model(path)
    with open(path) as f:
        mine = json.load(f)
    assert ref_keys <= set(mine), ref_keys - set(mine)
    b = M.load_model(path)
    assert np.array_equal(b._nan_bin_id, m._nan_bin_id)
    assert b.learning_rate == 0.0625
    assert np.array_equal(b.bin_edges, m.bin_edges)
    for ta, tb in zip(m.trees, b.trees):
        for i in range(7):
            assert np.array_equal(np.asarray(ta[i]), np.asarray(tb[i]))
    for k in ("_packed_features", "_packed_thresholds", "_packed_values", "_packed_left",
              "_packed_right", "_tree_offsets"):
        assert np.array_equal(getattr(m, k), getattr(b, k)), k


@pytest.mark.gpu
def test_loaded_reference_model_predicts_like_the_reference():
    d = np.load(os.path.join(GOLDEN, "model_ref_cfg3.npz"))
    _, _, Xte = fit_inputs("cfg3_small")
    m = _model_cls().load_model(REF_JSON)
    p = m.predict_proba(Xte)
    assert np.abs(p - d["proba_test_loaded"]).max() <= 1e-9
    assert np.abs(p - d["proba_test"]).max() <= 1e-9      # no NaN in config 3: same as before the reload


@pytest.mark.gpu
def test_round_trip_keeps_nan_bins(tmp_path):
    M = _model_cls()
    X, y, Xte = fit_inputs("cfg4_small")                  # 30 % NaN in every feature
    m = M(n_estimators=5, max_depth=6, n_bins=255, random_state=2, verbose=False).fit(X, y)
    path = str(tmp_path / "m.json")
    m.save_model(path)
    b = M.load_model(path)
    assert np.array_equal(b.predict_proba(Xte), m.predict_proba(Xte))
