"""Parity at the benchmark configurations' full sizes, on the GPU.

Each case fits ``HybridHistGBMNumbaV1_0_1`` through its public ``fit`` (GPU bin
edges and bins, every round on the device) on the seeded stand-in data at
the size the benchmark names, and compares with the reference's own fit of
the same data recorded by ``tests/golden/make_golden_full.py``:

* ``cfg4_d6``  config 4, 1,000,000 x 100 float32 (30 % NaN), depth 6, 205
  trees -- bench.py's workload and its 5 warm-up + 200 timed rounds;
* ``cfg4_d8``  the same data at max_depth 8, 200 trees;
* ``cfg2``     config 2, 284,807 x 30, balanced_sqrt, 500 trees;
* ``cfg3``     config 3, 50,000 x 20, balanced_sqrt, 300 trees;
* ``top257``   the reference's default constructor (n_bins 'auto' = 256, so
  257 bin ids per feature) on 20,000 x 30 with splits at threshold 255.

What must hold:

* bin edges, bin counts, NaN bins and the base score equal the reference's;
* every tree's topology (features, thresholds, children, node count) equals
  the reference's up to the first node where the engine's exact fixed-point
  arithmetic departs from it -- the fixture records that node (from the
  oracle's EXACT mode) and an audit showing it is an exact tie of the
  reference's own round inputs (two different splits with equal exact
  gains, which the reference breaks by float64 rounding noise); with no
  such node every tree must match;
* before that node, leaf values within 1e-6 and
  train losses within 1e-9 of the reference's; with no divergence also
  predict_proba on held-out rows within 1e-6;
* every tree, before and after the tie, equals the oracle's EXACT
  trajectory in topology, with leaf values within 1e-9 and losses within
  1e-9 (the engine's sums are exact; its gradients use CUDA's exp, which
  can differ from the C library's in the last bit).
"""
import numpy as np
import pytest

import audit as A
from helpers import golden

pytestmark = pytest.mark.gpu

CASES = ["cfg4_d6", "cfg4_d8", "cfg2", "cfg3", "top257"]


def _trees(d, prefix=""):
    out = []
    for t in range(int(d["n_trees"])):
        nc = int(d[prefix + "nc"][t])
        out.append(tuple(d[prefix + k][t] for k in ("tf", "tt", "tv", "tl", "tr")) + (nc, d[prefix + "sg"][t]))
    return out


def _data(name):
    from bsscl_gbm_b200 import datasets as D
    if name == "top257":
        X, y = D.top_bin()
        Xh, _ = D.top_bin(n=5_000, seed=22)
    elif name.startswith("cfg4"):
        X, y = D.config4(n=1_000_000)
        Xh, _ = D.config4(n=20_000, seed=13)
    elif name == "cfg2":
        X, y = D.config2()
        Xh, _ = D.config2(n=20_000, seed=11, n_pos=40)
    else:
        X, y = D.config3()
        Xh, _ = D.config3(n=20_000, seed=12)
    return X, y, Xh


def _params(d):
    import ast
    p = dict(ast.literal_eval(str(d["params"])))
    p.pop("data")
    return p


@pytest.mark.parametrize("name", CASES)
def test_full_size_fit_matches_reference(name):
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    d = golden("fit_full_" + name)
    X, y, Xh = _data(name)
    m = M(verbose=False, **_params(d)).fit(X, y)
    # resolved hyper-parameters, binning and base score
    assert (m.max_leaves, m.max_depth) == (int(d["max_leaves"]), int(d["max_depth"]))
    assert m.learning_rate == float(d["learning_rate"]) and m.subsample == float(d["subsample"])
    assert np.array_equal(m.feature_bin_counts, d["counts"])
    assert np.array_equal(m._nan_bin_id, d["nan_bin_id"])
    assert np.array_equal(m.bin_edges, d["edges"])
    assert m.base_score_ == float(d["base_score"])
    ref, ex = _trees(d), _trees(d, "exact_")
    assert len(m.trees) == len(ref)
    # against the reference: identical until the recorded exact tie
    div = A.first_divergence(ref, m.trees)
    if bool(d["has_div"]):
        assert str(d["audit_kind"]) in ("exact_tie", "same_partition")
        assert div == (int(d["div_tree"]), int(d["div_node"])), div
    else:
        assert div is None, div
    upto = len(ref) if div is None else div[0]
    for t in range(upto):
        nc = ref[t][5]
        assert np.abs(m.trees[t][2][:nc] - ref[t][2][:nc]).max() <= 1e-6, f"values tree {t}"
    loss = np.array(m.train_loss_history_)
    assert np.abs(loss[:upto] - d["train_loss"][:upto]).max(initial=0.0) <= 1e-9
    if div is None:
        assert np.abs(m.predict_proba(Xh) - d["proba_heldout"]).max() <= 1e-6
    # against the engine's exact arithmetic on the CPU (oracle EXACT mode): every tree
    assert A.first_divergence(ex, m.trees) is None
    for t in range(len(ex)):
        nc = ex[t][5]
        assert np.abs(m.trees[t][2][:nc] - ex[t][2][:nc]).max() <= 1e-9, f"EXACT values tree {t}"
    assert np.abs(loss - d["exact_train_loss"]).max() <= 1e-9
