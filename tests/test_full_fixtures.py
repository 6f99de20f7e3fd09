"""The full-size reference fixtures (tests/golden/fit_full_*.npz), checked on
the CPU: what the GPU parity tests at the benchmark sizes rely on.

* The oracle's EXACT trajectory recorded in each fixture leaves the
  reference's trees at the recorded node only, and the audit made there
  (exact rational gains of both splits on the reference's own round
  inputs) found an exact tie.
* The native sampler draws, at the full row counts, the reference's
  per-round row and feature samples (their SHA-256 hashes).
* Class weights and base score of the regenerated labels equal the
  reference's base score.
"""
import hashlib
import ast

import numpy as np
import pytest

import audit as A
import oracle as O
from helpers import golden

CASES = ["cfg4_d6", "cfg4_d8", "cfg2", "cfg3", "top257"]


def _trees(d, prefix=""):
    return [tuple(d[prefix + k][t] for k in ("tf", "tt", "tv", "tl", "tr")) + (int(d[prefix + "nc"][t]),
                                                                              d[prefix + "sg"][t])
            for t in range(int(d["n_trees"]))]


def _labels(name):
    from bsscl_gbm_b200 import datasets as D
    if name == "top257":
        return D.top_bin()[1], 20_000, 30
    if name.startswith("cfg4"):
        return D.config4(n=1_000_000)[1], 1_000_000, 100
    if name == "cfg2":
        return D.config2()[1], 284_807, 30
    return D.config3()[1], 50_000, 20


@pytest.mark.parametrize("name", CASES)
def test_exact_trajectory_leaves_the_reference_only_at_an_audited_tie(name):
    d = golden("fit_full_" + name)
    div = A.first_divergence(_trees(d), _trees(d, "exact_"))
    if bool(d["has_div"]):
        assert div == (int(d["div_tree"]), int(d["div_node"]))
        assert str(d["audit_kind"]) in ("exact_tie", "same_partition")
    else:
        assert div is None
        assert np.abs(d["exact_train_loss"] - d["train_loss"]).max() <= 1e-9


@pytest.mark.parametrize("name", CASES)
def test_sampler_and_base_score_at_full_size(name, built_lib):
    from bsscl_gbm_b200 import Sampler
    d = golden("fit_full_" + name)
    y, n, p = _labels(name)
    params = ast.literal_eval(str(d["params"]))
    w2 = O.class_weights(y, params.get("class_weight", "balanced_sqrt"))
    assert O.base_score(y, w2) == float(d["base_score"])
    s = Sampler(params["random_state"], n, p, int(n * float(d["subsample"])), int(p * float(d["colsample"])),
                True, True)
    for t in range(12):
        smp, _, feat = s.next(want_sample=True, want_mask=False)
        assert hashlib.sha256(smp.tobytes()).hexdigest() == str(d["sample_sha"][t]), f"round {t} rows"
        assert hashlib.sha256(np.ascontiguousarray(feat, np.int32).tobytes()).hexdigest() == str(d["feat_sha"][t])
    s.close()


def test_top257_fixture_has_257_bins_and_threshold_255_splits():
    """The reference's default constructor at p = 30: n_bins 256, so every
    feature holds 257 bin ids (0..256, E:2111-2127), and the reference
    chose threshold 255 (bin 256 alone on the right) more than once."""
    from bsscl_gbm_b200 import datasets as D
    d = golden("fit_full_top257")
    assert int(d["n_bins"]) == 256 and int(np.max(d["counts"])) == 257
    trees = _trees(d)
    n255 = sum(int(np.sum((t[0][:t[5]] >= 0) & (t[1][:t[5]] == 255))) for t in trees)
    assert n255 >= 10
    # the oracle's binning (the reference's _bin_features restated) gives the reference's uint16 ids
    X, _ = D.top_bin()
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], str(d["binning_strategy"]) == "hybrid")
    assert int(Xb.max()) == 256
    assert hashlib.sha256(Xb.astype(np.uint16).tobytes()).hexdigest() == str(d["X_bin_sha"])


def test_top257_oracle_ref_fit_equals_the_reference():
    """The oracle's REF mode on the 257-bin ids reproduces the reference's
    trees and losses (ties included): the restatement is pinned at bin 256."""
    from bsscl_gbm_b200 import datasets as D
    d = golden("fit_full_top257")
    X, y = D.top_bin()
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], str(d["binning_strategy"]) == "hybrid")
    res = O.fit_binary(Xb, y, d["counts"], n_estimators=int(d["n_trees"]), learning_rate=float(d["learning_rate"]),
                       max_leaves=int(d["max_leaves"]), max_depth=int(d["max_depth"]),
                       min_samples_leaf=int(d["min_samples_leaf"]), min_child_weight=float(d["min_child_weight"]),
                       reg_lambda=float(d["reg_lambda"]), gamma=float(d["gamma"]), subsample=float(d["subsample"]),
                       colsample=float(d["colsample"]), class_weight="balanced_sqrt", random_state=0,
                       mode=O.MODE_REF)
    assert A.first_divergence(_trees(d), res["trees"]) is None
    assert np.abs(np.asarray(res["train_loss"]) - d["train_loss"]).max() <= 1e-12
