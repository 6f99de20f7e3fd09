"""CUDA engine parity, through the C ABI (libgbm_b200.so), on a B200.

* gbm_build_tree on every golden tree case == the oracle's EXACT builder,
  bit for bit (topology, values, gains), and == the reference's topology.
* gbm_round, round after round: tree == oracle EXACT on the engine's own
  gradients (bit for bit), per-row leaf ids, F update and train loss.
* Full fits through the estimator vs the reference's recorded fits:
  identical trees until a divergence, which must be an exact tie; leaf
  values and predict_proba within 1e-6.
* Predict on a packed ensemble vs the reference's predict_all_trees_jit.
"""
import glob
import os

import numpy as np
import pytest

import audit as A
import oracle as O
from conftest import GOLDEN
from helpers import fit_inputs, fit_params, golden, golden_trees, same_topology

pytestmark = pytest.mark.gpu

TREE_CASES = sorted(os.path.basename(f)[5:-4] for f in glob.glob(os.path.join(GOLDEN, "tree_*.npz")))


def _params(max_leaves=63, max_depth=6, msl=5, mcw=1.0, lam=1.0, gamma=0.0, lr=0.1, policy="leaf"):
    from bsscl_gbm_b200 import GbmParams
    return GbmParams(float(lam), float(gamma), float(mcw), float(lr), int(msl), int(max_depth),
                     int(max_leaves), 0 if policy == "leaf" else 1, None)


def _cap(max_leaves, max_depth, policy):
    return 2 * max_leaves + 2 if policy == "leaf" else (1 << (max_depth + 1)) - 1


def _assert_tree_equal(a, b, what=""):
    nc = a[5]
    assert nc == b[5], f"{what}: node count {nc} vs {b[5]}"
    for i, k in [(0, "tf"), (1, "tt"), (2, "tv"), (3, "tl"), (4, "tr"), (6, "sg")]:
        x, y = np.asarray(a[i])[:nc], np.asarray(b[i])[:nc]
        assert np.array_equal(x, y), f"{what}: {k} differs at {np.nonzero(x != y)[0][:5]}"


@pytest.mark.parametrize("case", TREE_CASES)
def test_build_tree_matches_oracle_exact(engine, case):
    from bsscl_gbm_b200 import binning
    d = golden("tree_" + case)
    counts = d["counts"]
    Xb = d["X_bin"]
    n = Xb.shape[0]
    engine.upload_bins(binning.device_bins(Xb, counts), counts)
    mask = np.zeros(n, np.uint8)
    mask[d["sample_idx"]] = 1
    pol = str(d["policy"])
    kw = dict(max_leaves=int(d["max_leaves"]), max_depth=int(d["max_depth"]), msl=int(d["msl"]),
              mcw=float(d["mcw"]), lam=float(d["lam"]), gamma=float(d["gamma"]))
    t = engine.build_tree(d["g"], d["h"], mask, d["feat_idx"], _params(policy=pol, **kw),
                          _cap(kw["max_leaves"], kw["max_depth"], pol))
    S = engine.scale_bits()
    o = O.build_tree(Xb, d["g"], d["h"], d["sample_idx"], d["feat_idx"], counts, mode=O.MODE_EXACT,
                     scale_bits=S, policy=pol, **kw)
    O.post_prune(o[0], o[3], o[4], o[6], kw["gamma"], o[5])
    _assert_tree_equal(t, o, case)
    ref = (d["tf_pruned"], d["tt"], d["tv"], d["tl_pruned"], d["tr_pruned"], int(d["nc"]), d["sg"])
    assert same_topology(t, ref)
    nc = t[5]
    assert np.abs(t[2][:nc] - d["tv"][:nc]).max() <= 1e-9


@pytest.mark.parametrize("depth", [10, 14])
@pytest.mark.parametrize("case", ["basic", "few_bins", "tied", "nan_heavy", "leaves4", "gamma", "msl_big",
                                  "mcw_big"])
def test_build_tree_deep_matches_oracle_exact(engine, case, depth):
    """Depth 10 expands every level that the best-first loop can still reach
    (full speculation, with the nodes it can provably never split left out:
    a node is skipped once max_leaves - 1 splits are certain to come before
    it) and replays on the device; depth 14 ranks each level's expansions
    (capped at max_leaves - 1) and replays on the host, expanding on demand
    what the ranking left out.  The same bit-exact bar."""
    from bsscl_gbm_b200 import binning
    d = golden("tree_" + case)
    counts = d["counts"]
    Xb = d["X_bin"]
    n = Xb.shape[0]
    engine.upload_bins(binning.device_bins(Xb, counts), counts)
    mask = np.zeros(n, np.uint8)
    mask[d["sample_idx"]] = 1
    kw = dict(max_leaves=int(d["max_leaves"]), max_depth=depth, msl=int(d["msl"]),
              mcw=float(d["mcw"]), lam=float(d["lam"]), gamma=float(d["gamma"]))
    t = engine.build_tree(d["g"], d["h"], mask, d["feat_idx"], _params(**kw),
                          _cap(kw["max_leaves"], kw["max_depth"], "leaf"))
    o = O.build_tree(Xb, d["g"], d["h"], d["sample_idx"], d["feat_idx"], counts, mode=O.MODE_EXACT,
                     scale_bits=engine.scale_bits(), policy="leaf", **kw)
    O.post_prune(o[0], o[3], o[4], o[6], kw["gamma"], o[5])
    _assert_tree_equal(t, o, case)


def test_build_tree_empty_inbag(engine):
    """No in-bag rows: the root is a leaf with value -0/(0+lambda), like the reference."""
    from bsscl_gbm_b200 import binning
    d = golden("tree_basic")
    engine.upload_bins(binning.device_bins(d["X_bin"], d["counts"]), d["counts"])
    mask = np.zeros(d["X_bin"].shape[0], np.uint8)
    t = engine.build_tree(d["g"], d["h"], mask, d["feat_idx"], _params(), 128)
    assert t[5] == 1 and t[0][0] == -1 and t[2][0] == 0.0


def _cfg1_engine(engine, n=10_000):
    from bsscl_gbm_b200 import binning
    d = golden("fit_cfg1")
    X, y, _ = fit_inputs("cfg1")
    Xb = binning.bin_features(X, d["edges"], d["counts"], d["nan_bin_id"])
    w2 = O.class_weights(y, None)
    base = O.base_score(y, w2)
    engine.upload_bins(binning.device_bins(Xb, d["counts"]), d["counts"])
    engine.upload_labels(y.astype(np.uint8), w2, base, n_global=len(y))
    return d, Xb, y, w2, base


@pytest.mark.parametrize("policy", ["leaf", "level"])
def test_rounds_match_oracle_exact(engine, policy):
    from bsscl_gbm_b200 import Sampler
    d, Xb, y, w2, base = _cfg1_engine(engine)
    n, p = Xb.shape
    lr = 0.1
    kw = dict(max_leaves=31, max_depth=6 if policy == "leaf" else 5, msl=5, mcw=2.0, lam=1.0,
              gamma=0.0)
    prm = _params(lr=lr, policy=policy, **kw)
    cap = _cap(kw["max_leaves"], kw["max_depth"], policy)
    s = Sampler(0, n, p, int(n * 0.8), int(p * 0.8), True, True)
    F_prev = engine.get_F()
    assert np.all(F_prev == base)
    S = engine.scale_bits()
    y8 = y.astype(np.uint8)
    for r in range(6):
        g, h = engine.get_grad()
        og, oh = O.grad_hess(F_prev, y8, w2)
        # CUDA's exp and the C library's differ by at most an ulp or two
        assert np.abs(g - og).max() <= 1e-14 and np.abs(h - oh).max() <= 1e-14
        smp, mask, feat = s.next(want_sample=True, want_mask=True)
        tree, loss, leaf = engine.round(mask, feat, prm, cap, want_leaf=True)
        o = O.build_tree(Xb, g, h, smp, feat, d["counts"], mode=O.MODE_EXACT, scale_bits=S,
                         policy=policy, **kw)
        O.post_prune(o[0], o[3], o[4], o[6], kw["gamma"], o[5])
        _assert_tree_equal(tree, o, f"round {r}")
        nc = tree[5]
        assert np.array_equal(leaf, O.leaf_ids(Xb, tree[0][:nc], tree[1][:nc], tree[3][:nc],
                                               tree[4][:nc]))
        F = engine.get_F()
        assert np.array_equal(F, F_prev + lr * tree[2][leaf])
        assert abs(loss - O.logloss(F, y8)) <= 1e-12 * max(1.0, abs(loss))
        F_prev = F
    s.close()


@pytest.mark.parametrize("name", ["cfg1", "cfg1_level", "cfg2_small", "cfg3_small", "cfg4_small", "spw"])
def test_fit_matches_reference(name):
    """The estimator on the GPU vs the reference's own recorded fit."""
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    d = golden("fit_" + name)
    X, y, Xte = fit_inputs(name)
    m = M(verbose=False, **fit_params(d)).fit(X, y)
    assert m.base_score_ == float(d["base_score"])
    ref = golden_trees(d)
    assert len(m.trees) == len(ref)
    div = A.first_divergence(ref, m.trees)
    upto = len(ref) if div is None else div[0]
    for t in range(upto):
        nc = ref[t][5]
        assert np.abs(m.trees[t][2][:nc] - ref[t][2][:nc]).max() <= 1e-6, f"values tree {t}"
    if div is None:
        assert np.abs(m.predict_proba(Xte) - d["proba_test"]).max() <= 1e-6
        assert np.abs(np.array(m.train_loss_history_) - d["train_loss"]).max() <= 1e-9
        return
    # a divergence must be an exact tie of the reference's own round inputs
    t = div[0]
    assert f"r{t}_g" in d.files, f"divergence at tree {t} beyond the recorded rounds"
    from bsscl_gbm_b200 import binning
    Xb = binning.bin_features(X, d["edges"], d["counts"], d["nan_bin_id"])
    res = A.audit_node(Xb, d[f"r{t}_g"], d[f"r{t}_h"], d[f"r{t}_sample"], d["counts"], ref[t],
                       m.trees[t], div[1], float(d["reg_lambda"]), float(d["min_child_weight"]))
    assert A.explained(res), res


def test_monotone_fit_matches_reference():
    """monotone_constraints on four features: the device replay's clip after
    the post-prune (E:2450-2457, E:2461-2499) gives the reference's recorded
    fit (tests/golden/fit_mono.npz).  The oracle's EXACT arithmetic meets no
    tie on this fit (tests/test_oracle.py), so every tree must match."""
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    d = golden("fit_mono")
    X, y, Xte = fit_inputs("mono")
    m = M(verbose=False, **fit_params(d)).fit(X, y)
    ref = golden_trees(d)
    assert len(m.trees) == len(ref)
    assert A.first_divergence(ref, m.trees) is None
    for t in range(len(ref)):
        nc = ref[t][5]
        assert np.abs(m.trees[t][2][:nc] - ref[t][2][:nc]).max() <= 1e-6, f"values tree {t}"
    assert np.abs(m.predict_proba(Xte) - d["proba_test"]).max() <= 1e-6
    assert np.abs(np.array(m.train_loss_history_) - d["train_loss"]).max() <= 1e-9


def test_early_stopping_fit_matches_reference():
    """A validation set with early_stopping_rounds (E:2908-2935): the same
    best iteration, kept trees, loss histories and predict_proba as the
    reference's recorded fit (tests/golden/fit_early.npz).  Its stopping
    decisions are clear of rounding noise and EXACT arithmetic meets no tie
    on it (tests/test_oracle.py)."""
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    from helpers import early_inputs
    d = golden("fit_early")
    Xtr, ytr, Xva, yva, Xte = early_inputs()
    m = M(verbose=False, **fit_params(d)).fit(Xtr, ytr, X_val=Xva, y_val=yva)
    assert m.best_iteration_ == int(d["best_iteration"])
    assert m.n_trees_fitted_ == int(d["n_trees_fitted"])
    ref = golden_trees(d)
    assert len(m.trees) == len(ref)
    assert A.first_divergence(ref, m.trees) is None
    for t in range(len(ref)):
        nc = ref[t][5]
        assert np.abs(m.trees[t][2][:nc] - ref[t][2][:nc]).max() <= 1e-6, f"values tree {t}"
    assert np.abs(np.array(m.val_loss_history_) - d["val_loss"]).max() <= 1e-9
    assert np.abs(np.array(m.train_loss_history_) - d["train_loss"]).max() <= 1e-9
    assert np.abs(m.predict_proba(Xte) - d["proba_test"]).max() <= 1e-6


def test_fit_is_deterministic():
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    X, y, Xte = fit_inputs("cfg3_small")
    kw = dict(n_estimators=8, max_depth=6, class_weight="balanced_sqrt", n_bins=255,
              random_state=5, verbose=False)
    a = M(**kw).fit(X, y)
    b = M(**kw).fit(X, y)
    for ta, tb in zip(a.trees, b.trees):
        _assert_tree_equal(ta, tb)
    assert np.array_equal(a.predict_proba(Xte), b.predict_proba(Xte))


def test_predict_matches_reference_ensemble(engine):
    d = golden("predict_ensemble")
    packed = {k: d[k] for k in ("features", "thresholds", "values", "left", "right", "offsets")}
    F, P = engine.predict(d["X_bin"].astype(np.uint8), packed, 40, float(d["lr"]), 0.0)
    assert np.abs(F - d["F"]).max() <= 1e-12
    assert np.abs(P - 1.0 / (1.0 + np.exp(-d["F"]))).max() <= 1e-12


def test_predict_proba_matches_oracle_random_forest(engine):
    """A larger random ensemble (full depth-8 trees) against the oracle."""
    from bsscl_gbm_b200 import datasets as D
    ens = D.config5_ensemble(n_trees=60, depth=8, p=40, seed=9)
    Xb = np.random.default_rng(9).integers(0, 255, size=(50_000, 40)).astype(np.uint8)
    F, _ = engine.predict(Xb, ens, 60, 0.08, -1.5, want_proba=False)
    Fo = O.predict_packed(Xb, ens, 60, 0.08) + (-1.5)
    assert np.abs(F - Fo).max() <= 1e-12


def test_round_sampled_equals_round_with_mask(engine):
    """gbm_round_sampled (device-built mask) == gbm_round with the same draw."""
    from bsscl_gbm_b200 import Sampler
    d, Xb, y, w2, base = _cfg1_engine(engine)
    n, p = Xb.shape
    prm = _params(max_leaves=31, max_depth=6, mcw=2.0)
    s1 = Sampler(0, n, p, int(n * 0.8), int(p * 0.8), True, True, look_ahead=2)
    trees_a = []
    for _ in range(4):
        t, _, _ = engine.round_sampled(s1, 0, prm, 64)
        trees_a.append(t)
    Fa = engine.get_F()
    s1.close()
    engine.upload_labels(y.astype(np.uint8), w2, base, n_global=len(y))
    s2 = Sampler(0, n, p, int(n * 0.8), int(p * 0.8), True, True, look_ahead=0)
    for r in range(4):
        _, mask, feat = s2.next(want_sample=False, want_mask=True)
        t, _, _ = engine.round(mask, feat, prm, 64)
        _assert_tree_equal(trees_a[r], t, f"round {r}")
    assert np.array_equal(engine.get_F(), Fa)
    s2.close()


@pytest.mark.parametrize("policy,depth,leaves", [("leaf", 6, 31), ("level", 5, 31), ("leaf", 8, 15),
                                                 ("leaf", 11, 31)])
def test_fit_rounds_equals_round_sampled(engine, policy, depth, leaves):
    """gbm_fit_rounds (rounds queued back to back, several in flight) gives
    the trees, losses and F of the same number of gbm_round_sampled calls;
    depth 11 takes the one-by-one path (host replay)."""
    from bsscl_gbm_b200 import Sampler
    d, Xb, y, w2, base = _cfg1_engine(engine)
    n, p = Xb.shape
    prm = _params(max_leaves=leaves, max_depth=depth, mcw=2.0, policy=policy)
    cap = _cap(leaves, depth, policy)
    rounds = 9
    s1 = Sampler(3, n, p, int(n * 0.7), int(p * 0.6), True, True, look_ahead=2)
    ref = [engine.round_sampled(s1, 0, prm, cap)[:2] for _ in range(rounds)]
    Fa = engine.get_F()
    s1.close()
    engine.upload_labels(y.astype(np.uint8), w2, base, n_global=len(y))
    s2 = Sampler(3, n, p, int(n * 0.7), int(p * 0.6), True, True, look_ahead=2)
    got = engine.fit_rounds(s2, 0, prm, cap, 5) + engine.fit_rounds(s2, 0, prm, cap, rounds - 5)
    s2.close()
    for r in range(rounds):
        _assert_tree_equal(ref[r][0], got[r][0], f"round {r}")
        assert ref[r][1] == got[r][1]
    assert np.array_equal(engine.get_F(), Fa)


def test_device_row_shuffle_at_scale(engine):
    """300k rows: the rounds whose in-bag rows come from the device-side
    shuffle (gbm_round_sampled) equal the rounds given the host sampler's
    masks (gbm_round), tree for tree and in F."""
    from bsscl_gbm_b200 import Sampler
    rng = np.random.default_rng(4)
    n, p = 300_000, 20
    Xb = rng.integers(0, 64, size=(n, p)).astype(np.uint8)
    counts = np.full(p, 64, np.int32)
    y = (rng.random(n) < 0.3).astype(np.uint8)
    w2 = O.class_weights(y, None)
    base = O.base_score(y, w2)
    engine.upload_bins(Xb, counts)
    engine.upload_labels(y, w2, base, n_global=n)
    prm = _params(max_leaves=15, max_depth=4)
    s1 = Sampler(21, n, p, int(n * 0.6), 12, True, True, look_ahead=3)
    a = [engine.round_sampled(s1, 0, prm, 32)[0] for _ in range(3)]
    Fa = engine.get_F()
    s1.close()
    engine.upload_labels(y, w2, base, n_global=n)
    s2 = Sampler(21, n, p, int(n * 0.6), 12, True, True, look_ahead=0)
    for r in range(3):
        _, mask, feat = s2.next(want_sample=False, want_mask=True)
        t, _, _ = engine.round(mask, feat, prm, 32)
        _assert_tree_equal(a[r], t, f"round {r}")
    assert np.array_equal(engine.get_F(), Fa)
    s2.close()


def _scale_data(n, p, seed):
    """Bins like config 4's: quantile-uniform columns, few-level columns and a
    NaN bin on 30 % of the rows of every third column."""
    rng = np.random.default_rng(seed)
    counts = np.empty(p, np.int32)
    Xb = np.empty((n, p), np.uint8)
    for j in range(p):
        if j % 7 == 3:                                   # integer levels
            lv = int(rng.integers(2, 12))
            Xb[:, j] = rng.integers(0, lv, n)
            counts[j] = lv
        else:
            Xb[:, j] = rng.integers(0, 255, n)
            counts[j] = 256 if j % 3 == 0 else 255
            if j % 3 == 0:
                Xb[rng.random(n) < 0.3, j] = 255         # the NaN bin
    logit = (Xb[:, 0].astype(np.float64) - 128) / 40 + (Xb[:, 3] == 1) - 1.5
    y = (rng.random(n) < 1 / (1 + np.exp(-logit))).astype(np.uint8)
    return Xb, counts, y


@pytest.mark.parametrize("n,p,drop", [(600_000, 40, range(16, 32)), (250_000, 100, range(96, 100))])
def test_rounds_match_oracle_exact_at_scale(engine, n, p, drop):
    """Full-size launches (equal-work histogram CTAs spanning several nodes
    and feature blocks, nodes over 16k rows, a feature block with no
    selected feature) stay bit-exact with the oracle's EXACT builder."""
    Xb, counts, y = _scale_data(n, p, seed=n)
    w2 = O.class_weights(y, "balanced_sqrt")
    base = O.base_score(y, w2)
    engine.upload_bins(Xb, counts)
    engine.upload_labels(y, w2, base, n_global=n)
    kw = dict(max_leaves=63, max_depth=6, msl=5, mcw=3.0, lam=1.0, gamma=0.0)
    prm = _params(lr=0.08, **kw)
    rng = np.random.default_rng(7)
    keep = np.array([j for j in range(p) if j not in set(drop)])
    S = engine.scale_bits()
    for r in range(2):
        g, h = engine.get_grad()
        smp = rng.choice(n, int(0.75 * n), replace=False)
        mask = np.zeros(n, np.uint8)
        mask[smp] = 1
        feat = np.sort(rng.choice(keep, int(0.7 * len(keep)), replace=False)).astype(np.int32)
        tree, _, _ = engine.round(mask, feat, prm, 128)
        o = O.build_tree(Xb, g, h, smp, feat, counts, mode=O.MODE_EXACT, scale_bits=S, **kw)
        O.post_prune(o[0], o[3], o[4], o[6], kw["gamma"], o[5])
        _assert_tree_equal(tree, o, f"round {r}")


def _row_hash(seed, rnd, rows):
    """gbm_row_hash (csrc/gbm_common.cuh) restated with NumPy's wrapping uint64."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + np.uint64(rnd) * np.uint64(0xD1B54A32D192ED03) + \
            rows.astype(np.uint64) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def test_device_sampler_rows_are_the_documented_hash(engine):
    """The throughput-mode sampler (gbm_sampler_create_device): round r's
    in-bag rows are those whose gbm_row_hash(seed, r, row) < subsample *
    2^64, and its features are the reference stream's feature draws alone
    (a host sampler with row subsampling off gives the same).  Every tree
    equals the oracle's EXACT tree on exactly those rows and features."""
    from bsscl_gbm_b200 import Sampler
    d, Xb, y, w2, base = _cfg1_engine(engine)
    n, p = Xb.shape
    seed, frac, nfeat = 7, 0.6, int(p * 0.8)
    s = Sampler.device(seed, n, p, frac, nfeat, True)
    twin = Sampler(seed, n, p, n, nfeat, False, True)
    dseed = (0x9E3779B97F4A7C15 * (seed + 1)) & 0xFFFFFFFFFFFFFFFF
    thr = np.uint64(int(np.ldexp(frac, 64)))
    kw = dict(max_leaves=31, max_depth=6, msl=5, mcw=2.0, lam=1.0, gamma=0.0)
    prm = _params(lr=0.1, **kw)
    S = engine.scale_bits()
    for r in range(4):
        g, h = engine.get_grad()
        tree, loss, leaf = engine.round_sampled(s, 0, prm, 64, want_leaf=True)
        rows = np.flatnonzero(_row_hash(dseed, r, np.arange(n)) < thr).astype(np.int64)
        assert abs(len(rows) - frac * n) < 5 * np.sqrt(n)
        _, _, feat = twin.next(want_sample=False, want_mask=False)
        o = O.build_tree(Xb, g, h, rows, feat, d["counts"], mode=O.MODE_EXACT, scale_bits=S, **kw)
        O.post_prune(o[0], o[3], o[4], o[6], kw["gamma"], o[5])
        _assert_tree_equal(tree, o, f"round {r}")
    s.close()
    twin.close()
