"""The CPU oracle pinned against the reference's own outputs (tests/golden).

REF mode must reproduce the reference bit-for-bit (trees, values, gains,
bins, sampler-driven fits).  EXACT mode (the engine's arithmetic) must give
the same topology wherever the reference's choice is not an exact tie, and
every divergence must be explained by the exact-rational tie audit.
"""
import glob
import os

import numpy as np
import pytest

import audit as A
import oracle as O
from conftest import GOLDEN
from helpers import (engine_scale_bits, fit_inputs, golden, golden_trees, oracle_fit_kwargs,
                     same_topology)

TREE_CASES = sorted(os.path.basename(f)[5:-4] for f in glob.glob(os.path.join(GOLDEN, "tree_*.npz")))
BIN_CASES = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "bin_*.npz")))


def _tree_kwargs(d):
    return dict(max_leaves=int(d["max_leaves"]), max_depth=int(d["max_depth"]), msl=int(d["msl"]),
                mcw=float(d["mcw"]), lam=float(d["lam"]), gamma=float(d["gamma"]),
                policy=str(d["policy"]))


@pytest.mark.parametrize("case", TREE_CASES)
def test_ref_builder_bit_exact(case):
    d = golden("tree_" + case)
    tf, tt, tv, tl, tr, nc, sg = O.build_tree(d["X_bin"], d["g"], d["h"], d["sample_idx"],
                                              d["feat_idx"], d["counts"], **_tree_kwargs(d))
    assert nc == int(d["nc"])
    for a, k in [(tf, "tf"), (tt, "tt"), (tv, "tv"), (tl, "tl"), (tr, "tr"), (sg, "sg")]:
        assert np.array_equal(a, d[k]), k
    O.post_prune(tf, tl, tr, sg, float(d["gamma"]), nc)
    assert np.array_equal(tf, d["tf_pruned"])
    leaf = O.leaf_ids(d["X_bin"], tf[:nc], tt[:nc], tl[:nc], tr[:nc])
    assert np.array_equal(leaf, d["leaf_of_row"])


@pytest.mark.parametrize("case", TREE_CASES)
def test_exact_builder_topology(case):
    d = golden("tree_" + case)
    m = max(np.abs(d["g"]).max(), np.abs(d["h"]).max())
    S = engine_scale_bits(m)
    t = O.build_tree(d["X_bin"], d["g"], d["h"], d["sample_idx"], d["feat_idx"], d["counts"],
                     mode=O.MODE_EXACT, scale_bits=S, **_tree_kwargs(d))
    ref = (d["tf"], d["tt"], d["tv"], d["tl"], d["tr"], int(d["nc"]), d["sg"])
    if not same_topology(t, ref):
        div = A.first_divergence([ref], [t])
        res = A.audit_node(d["X_bin"], d["g"], d["h"], d["sample_idx"], d["counts"], ref, t,
                           div[1], float(d["lam"]), float(d["mcw"]))
        assert A.explained(res), res
    else:
        nc = t[5]
        assert np.abs(t[2][:nc] - d["tv"][:nc]).max() < 1e-9


@pytest.mark.parametrize("case", BIN_CASES)
def test_ref_binning_bit_exact(case):
    d = golden(case)
    Xb = O.bin_matrix(d["X"], d["edges"], d["counts"], d["nan_bin_id"], str(d["strategy"]) == "hybrid")
    assert np.array_equal(Xb, d["X_bin"])


def test_ref_predict_ensemble():
    d = golden("predict_ensemble")
    packed = {k: d[k] for k in ("features", "thresholds", "values", "left", "right", "offsets")}
    F = O.predict_packed(d["X_bin"], packed, 40, float(d["lr"]))
    assert np.abs(F - d["F"]).max() < 1e-12


def _binned(name, d):
    from bsscl_gbm_b200 import binning
    X, y, _ = fit_inputs(name)
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"],
                      str(d["binning_strategy"]) == "hybrid")
    return Xb, y


@pytest.mark.parametrize("name", ["cfg1", "cfg1_level", "cfg2_small", "cfg3_small", "cfg4_small"])
def test_ref_fit_bit_exact(name):
    """The oracle's boosting loop (NumPy sampler + REF builder) == the reference's fit."""
    d = golden("fit_" + name)
    Xb, y = _binned(name, d)
    import hashlib
    assert hashlib.sha256(Xb.astype(np.uint16).tobytes()).hexdigest() == str(d["X_bin_sha"])
    rec = []
    r = O.fit_binary(Xb, y, d["counts"], mode=O.MODE_REF, record=rec, **oracle_fit_kwargs(d))
    assert r["base_score"] == float(d["base_score"])
    for t, (a, b) in enumerate(zip(r["trees"], golden_trees(d))):
        assert same_topology(a, b), f"tree {t}"
        nc = a[5]
        assert np.abs(a[2][:nc] - b[2][:nc]).max() < 1e-12, f"values tree {t}"
    for t, rr in enumerate(rec):
        assert hashlib.sha256(rr["sample"].tobytes()).hexdigest() == str(d["sample_sha"][t])
    assert np.abs(r["train_loss"] - d["train_loss"]).max() < 1e-12


@pytest.mark.parametrize("name", ["cfg1", "cfg1_level", "cfg2_small", "cfg3_small", "cfg4_small", "spw"])
def test_exact_fit_ties_explained(name):
    """EXACT-mode fit: same trees as the reference up to the first divergence,
    and that divergence is an exact (or sub-resolution) tie."""
    d = golden("fit_" + name)
    Xb, y = _binned(name, d)
    kw = oracle_fit_kwargs(d)
    rec = []
    ref = O.fit_binary(Xb, y, d["counts"], mode=O.MODE_REF, record=rec, **kw)
    S = engine_scale_bits(ref["w2"].max())
    ex = O.fit_binary(Xb, y, d["counts"], mode=O.MODE_EXACT, scale_bits=S, **kw)
    div = A.first_divergence(ref["trees"], ex["trees"])
    if div is None:
        return
    t, _ = div
    rr = rec[t]
    te = O.build_tree(Xb, rr["g"], rr["h"], rr["sample"], rr["feat"], d["counts"],
                      max_leaves=kw["max_leaves"], max_depth=kw["max_depth"],
                      msl=kw["min_samples_leaf"], mcw=kw["min_child_weight"], lam=kw["reg_lambda"],
                      gamma=kw["gamma"], mode=O.MODE_EXACT, scale_bits=S, policy=kw["grow_policy"])
    O.post_prune(te[0], te[3], te[4], te[6], kw["gamma"], te[5])
    dv = A.first_divergence([ref["trees"][t]], [te])
    assert dv is not None
    res = A.audit_node(Xb, rr["g"], rr["h"], rr["sample"], d["counts"], ref["trees"][t], te, dv[1],
                       kw["reg_lambda"], kw["min_child_weight"])
    assert A.explained(res), res


def test_i128_conversion_rounds_to_nearest():
    """The oracle's 128-bit -> float64 conversion rounds to nearest-even, like
    Python's int -> float (and like the engine's device conversion)."""
    rng = np.random.default_rng(0)
    vals = [0, 1, -1, 2**53 + 1, 2**64 + 2**11, -(2**100) - 2**47 - 1, 2**126 - 1, -(2**126)]
    for _ in range(2000):
        bits = int(rng.integers(1, 126))
        v = int(rng.integers(0, 2**62)) << max(0, bits - 62)
        v |= int(rng.integers(0, 2**min(bits, 62)))
        vals.append(v if rng.random() < 0.5 else -v)
        vals.append((1 << bits) + (1 << max(0, bits - 53)))   # exact halfway cases
    for v in vals:
        assert O.i128_to_double(v) == float(v), v


def test_ref_multiclass_fit_bit_exact():
    """The oracle's multi-class loop (REF builder) == the reference's _fit_multiclass."""
    import hashlib
    from helpers import golden_mc_trees, mc_fit_kwargs
    d = golden("fit_mc")
    X, y, _ = fit_inputs("mc")
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    assert hashlib.sha256(Xb.astype(np.uint16).tobytes()).hexdigest() == str(d["X_bin_sha"])
    K = int(d["n_classes"])
    rec = []
    r = O.fit_multiclass(Xb, y, d["counts"], K, mode=O.MODE_REF, record=rec, **mc_fit_kwargs(d))
    ref = golden_mc_trees(d)
    for k in range(K):
        for t, (a, b) in enumerate(zip(r["trees"][k], ref[k])):
            assert same_topology(a, b), f"class {k} tree {t}"
            nc = a[5]
            assert np.abs(a[2][:nc] - b[2][:nc]).max() < 1e-12, f"values class {k} tree {t}"
    for t, rr in enumerate(rec):
        assert hashlib.sha256(rr["sample"].tobytes()).hexdigest() == str(d["sample_sha"][t])
    for t in range(3):
        for k in range(K):
            assert np.array_equal(rec[t]["g"][k], d[f"r{t}_k{k}_g"]), (t, k)
            assert np.array_equal(rec[t]["h"][k], d[f"r{t}_k{k}_h"]), (t, k)
    assert np.abs(r["train_loss"] - d["train_loss"]).max() < 1e-12


@pytest.mark.parametrize("loss", ["mse", "mae"])
def test_ref_regression_fit_bit_exact(loss):
    """The oracle's regression loop (REF builder) == the reference's _fit_regression."""
    import hashlib
    from helpers import golden_trees, reg_fit_kwargs
    d = golden(f"fit_reg_{loss}")
    X, y, _ = fit_inputs("reg")
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    assert hashlib.sha256(Xb.astype(np.uint16).tobytes()).hexdigest() == str(d["X_bin_sha"])
    rec = []
    r = O.fit_regression(Xb, y, d["counts"], loss=loss, mode=O.MODE_REF, record=rec, **reg_fit_kwargs(d))
    assert r["init_score"] == float(d["init_score"])
    for t, (a, b) in enumerate(zip(r["trees"], golden_trees(d))):
        assert same_topology(a, b), f"tree {t}"
        nc = a[5]
        assert np.abs(a[2][:nc] - b[2][:nc]).max() < 1e-9 * max(1.0, np.abs(b[2][:nc]).max()), f"values {t}"
    for t, rr in enumerate(rec):
        assert hashlib.sha256(rr["sample"].tobytes()).hexdigest() == str(d["sample_sha"][t])
    for t in range(3):
        assert np.array_equal(rec[t]["g"], d[f"r{t}_g"])
    assert np.abs(r["train_loss"] - d["train_loss"]).max() <= 1e-9 * np.abs(d["train_loss"]).max()


def test_ref_monotone_fit_bit_exact():
    """The oracle's loop with the monotone clip (E:2461-2499 after the
    post-prune, E:2450-2457) == the reference's fit with
    monotone_constraints on four features (tests/golden/fit_mono.npz)."""
    d = golden("fit_mono")
    Xb, y = _binned("mono", d)
    r = O.fit_binary(Xb, y, d["counts"], mode=O.MODE_REF, monotone=d["mono"], **oracle_fit_kwargs(d))
    assert r["base_score"] == float(d["base_score"])
    clipped = 0
    for t, (a, b) in enumerate(zip(r["trees"], golden_trees(d))):
        assert same_topology(a, b), f"tree {t}"
        nc = a[5]
        assert np.abs(a[2][:nc] - b[2][:nc]).max() < 1e-12, f"values tree {t}"
        for k in range(nc):   # splits whose children the clip made equal
            f = int(b[0][k])
            if f >= 0 and d["mono"][f] != 0 and abs(b[2][b[3][k]] - b[2][b[4][k]]) == 0.0:
                clipped += 1
    assert clipped > 0        # the fixture exercises the clip
    assert np.abs(r["train_loss"] - d["train_loss"]).max() < 1e-12


def test_exact_monotone_fit_has_no_tie():
    """The engine's fixed-point arithmetic (EXACT mode) gives every tree of
    the monotone fit as the reference does, so the GPU test of this fit
    compares every tree."""
    from helpers import engine_scale_bits
    d = golden("fit_mono")
    Xb, y = _binned("mono", d)
    kw = oracle_fit_kwargs(d)
    ref = O.fit_binary(Xb, y, d["counts"], mode=O.MODE_REF, monotone=d["mono"], **kw)
    ex = O.fit_binary(Xb, y, d["counts"], mode=O.MODE_EXACT, scale_bits=engine_scale_bits(ref["w2"].max()),
                      monotone=d["mono"], **kw)
    assert A.first_divergence(golden_trees(d), ex["trees"]) is None


def _early_fit(mode):
    """The oracle's loop run for the rounds the reference ran, the validation
    loss after each (E:2908-2916), and the reference's stopping rule
    (E:2924-2935) restated: (trees kept, best iteration, val losses)."""
    from helpers import early_inputs, val_loss, engine_scale_bits
    d = golden("fit_early")
    Xtr, ytr, Xva, yva, _ = early_inputs()
    hyb = str(d["binning_strategy"]) == "hybrid"
    Xb = O.bin_matrix(Xtr, d["edges"], d["counts"], d["nan_bin_id"], hyb)
    Xvb = O.bin_matrix(Xva, d["edges"], d["counts"], d["nan_bin_id"], hyb)
    kw = oracle_fit_kwargs(d)
    kw["n_estimators"] = len(d["val_loss"])
    S = None
    if mode == O.MODE_EXACT:
        w2 = O.class_weights(np.asarray(ytr), kw["class_weight"])
        S = engine_scale_bits(w2.max())
    r = O.fit_binary(Xb, ytr, d["counts"], mode=mode, scale_bits=S, **kw)
    F = np.full(len(yva), r["base_score"])
    losses, best, best_it, bad = [], np.inf, 0, 0
    for m, (tf, tt, tv, tl, tr, nc, sg) in enumerate(r["trees"]):
        F += kw["learning_rate"] * tv[O.leaf_ids(Xvb, tf, tt, tl, tr)]
        v = val_loss(yva, F)
        losses.append(v)
        if v < best:
            best, best_it, bad = v, m, 0
        else:
            bad += 1
            if bad >= 5:
                break
    return r["trees"][:best_it + 1], best_it, np.array(losses), d


@pytest.mark.parametrize("mode", [O.MODE_REF, O.MODE_EXACT])
def test_early_stopping_fit(mode):
    """REF and EXACT arithmetic both reproduce the reference's early-stopped
    fit: the same validation losses (to 1e-12), the same best iteration and
    kept trees.  Each stopping decision is clear of rounding noise, so the
    GPU test of this fit compares the same decisions."""
    trees, best_it, losses, d = _early_fit(mode)
    assert best_it == int(d["best_iteration"]) and len(trees) == int(d["n_trees"])
    assert len(losses) == len(d["val_loss"])
    assert np.abs(losses - d["val_loss"]).max() < 1e-12
    for t, (a, b) in enumerate(zip(trees, golden_trees(d))):
        assert same_topology(a, b), f"tree {t}"
        assert np.abs(a[2][:a[5]] - b[2][:b[5]]).max() < 1e-12, f"values tree {t}"
    run_best = np.minimum.accumulate(d["val_loss"])
    margins = np.abs(d["val_loss"][1:] - run_best[:-1])
    assert margins.min() > 1e-9


def test_spw_weighted_edges_match_reference():
    """scale_pos_weight=3 with objective='binary': the host's weighted bin
    edges (the reference's _build_bin_edges with sample_weight, E:3211-3216)
    equal the reference's, and so do the class weights (E:2572-2577)."""
    from bsscl_gbm_b200 import binning
    d = golden("fit_spw")
    X, y, _ = fit_inputs("spw")
    sw = np.ones(len(y))
    sw[y == 1] = 3.0
    e, c, nb = binning.build_bin_edges(X, int(d["n_bins"]), None, sw)
    assert np.array_equal(e, d["edges"]) and np.array_equal(c, d["counts"]) and np.array_equal(nb, d["nan_bin_id"])
    assert np.array_equal(O.class_weights(y, "balanced_sqrt", 3.0, "binary"), [1.0, 3.0])
    assert np.array_equal(O.class_weights(y, "balanced_sqrt", 3.0, "auto"),
                          O.class_weights(y, "balanced_sqrt"))   # 'auto' ignores it (E:2572)


def test_ref_spw_fit_bit_exact():
    """The oracle's loop with scale_pos_weight=3 and objective='binary' (the
    class weights of E:2572-2577) == the reference's fit; its sampler matches
    the recorded rounds."""
    d = golden("fit_spw")
    Xb, y = _binned("spw", d)
    rec = []
    r = O.fit_binary(Xb, y, d["counts"], mode=O.MODE_REF, record=rec, **oracle_fit_kwargs(d))
    assert r["base_score"] == float(d["base_score"])
    for t, (a, b) in enumerate(zip(r["trees"], golden_trees(d))):
        assert same_topology(a, b), f"tree {t}"
        assert np.abs(a[2][:a[5]] - b[2][:b[5]]).max() < 1e-12, f"values tree {t}"
    for t in range(4):
        assert np.array_equal(rec[t]["sample"], d[f"r{t}_sample"]) and np.array_equal(rec[t]["feat"], d[f"r{t}_feat"])
        # g, h to the last bits of exp (NumPy's SIMD exp vs the C library's)
        assert np.allclose(rec[t]["g"], d[f"r{t}_g"], rtol=1e-14, atol=0)
        assert np.allclose(rec[t]["h"], d[f"r{t}_h"], rtol=1e-14, atol=0)
    assert np.abs(r["train_loss"] - d["train_loss"]).max() < 1e-12


def _nan_like_high_case(seed=21, n=6000):
    """Feature 0: NaN in 30 % of rows, whose labels follow the rows with the
    highest values -- the split that sends NaN right separates the classes,
    the reference's NaN-left rule cannot."""
    from bsscl_gbm_b200 import binning
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, 4))
    y = (X[:, 0] > 0.8).astype(np.int64)
    nan = rng.random(n) < 0.3
    y[nan] = (rng.random(nan.sum()) < 0.9).astype(np.int64)
    X[nan, 0] = np.nan
    X[:, 1:] += 0.3 * y[:, None] * rng.random((n, 3))
    e, c, nb = binning.build_bin_edges(X, 64)
    Xb = binning.bin_features(X, e, c, nb)
    return Xb, y, c, nb


def test_oracle_learns_nan_right_where_it_gains_more():
    """With nan_bin_id (the engine's nan_direction) the root splits feature 0
    sending NaN right, with a larger gain than the best NaN-left split; that
    split's rows go as goes_left says; without nan_bin_id the tree is the
    reference's (no direction bits)."""
    Xb, y, counts, nanb = _nan_like_high_case()
    assert nanb[0] == 0
    w2 = O.class_weights(y, None)
    F = np.full(len(y), O.base_score(y, w2))
    g, h = O.grad_hess(F, y.astype(np.uint8), w2)
    sidx = np.arange(len(y), dtype=np.int64)
    fidx = np.arange(4, dtype=np.int32)
    kw = dict(max_leaves=8, max_depth=3, msl=5, mcw=1.0, lam=1.0, mode=O.MODE_EXACT, scale_bits=40)
    t0 = O.build_tree(Xb, g, h, sidx, fidx, counts, **kw)
    t1 = O.build_tree(Xb, g, h, sidx, fidx, counts, nan_bin_id=nanb, **kw)
    assert np.all((np.asarray(t0[1][:t0[5]]) >> 32) == 0)
    thr, nr = O.split_nan_right(t1[1])
    assert t1[0][0] == 0 and nr[0] == 1 and thr[0] >= 1
    assert t1[6][0] > t0[6][0]
    leaf = O.leaf_ids(Xb, t1[0], t1[1], t1[3], t1[4])
    b0 = Xb[:, 0].astype(np.int64)
    went_left = np.isin(leaf, _subtree(t1, int(t1[3][0])))
    assert np.array_equal(went_left, (b0 >= 1) & (b0 <= thr[0]))


def _subtree(t, k):
    out, stack = [], [k]
    while stack:
        u = stack.pop()
        out.append(u)
        if t[0][u] >= 0:
            stack += [int(t[3][u]), int(t[4][u])]
    return out
