"""Binning on the GPU, through the C ABI, on a B200.

* gbm_bin_edges == the reference's own _build_bin_edges output recorded in
  the golden fixtures (edges, bin counts, NaN bins), and gbm_bin_features ==
  its _bin_features ids, for float32/float64, 'standard'/'hybrid', n_bins
  255/254/32, NaN columns and integer levels.
* The same against the host restatement (NumPy's own unique/percentile)
  on matrices built to hit every branch: constant and all-NaN columns,
  signed zeros, values below 1e-8 (the float32 e[-1] + 1e-8 step), more
  distinct values than bins with heavy ties, infinities (NaN edges from
  np.percentile), huge magnitudes, n_bins down to 2.
* predict from raw rows (bins made on the GPU) == predict from host bins.
* The estimator's fit on the GPU-binned matrix == its fit on host bins.
"""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN
from helpers import fit_inputs, golden

pytestmark = pytest.mark.gpu

BIN_CASES = sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "bin_*.npz")))
FIT_CASES = ["cfg1", "cfg2_small", "cfg3_small", "cfg4_small"]


def _assert_ids(got, want, X, e, c, what=""):
    bad = np.argwhere(got != want)
    if len(bad):
        i, j = bad[0]
        k = int(want[i, j])
        raise AssertionError(
            f"{what}: {len(bad)} ids differ in columns {np.unique(bad[:, 1]).tolist()}; first at "
            f"({i}, {j}): x={X[i, j]!r} got {got[i, j]} want {k}, count {c[j]}, "
            f"edges[{max(0, k - 2)}:{k + 3}]={e[j][max(0, k - 2):k + 3].tolist()}")


def _assert_edges(e, c, nb, want_e, want_c, want_nb, what=""):
    assert np.array_equal(c, want_c), f"{what}: counts differ at {np.nonzero(c != want_c)[0][:5]}"
    assert np.array_equal(nb, want_nb), f"{what}: NaN bins differ"
    assert e.shape == want_e.shape, f"{what}: edges shape {e.shape} vs {want_e.shape}"
    bad = ~((e == want_e) | (np.isnan(e) & np.isnan(want_e)))
    assert not bad.any(), f"{what}: edges differ at {np.argwhere(bad)[:5].tolist()}"


@pytest.mark.parametrize("case", BIN_CASES)
def test_edges_and_ids_match_reference(engine, case):
    d = golden(case)
    e, c, nb = engine.bin_edges(d["X"], int(d["n_bins"]))
    _assert_edges(e, c, nb, d["edges"], d["counts"], d["nan_bin_id"], case)
    ids = engine.bin_features(d["X"], e, c, nb)
    assert np.array_equal(ids, d["X_bin"])


@pytest.mark.parametrize("name", FIT_CASES)
def test_edges_match_reference_fit(engine, name):
    import hashlib
    d = golden("fit_" + name)
    X, _, _ = fit_inputs(name)
    if not np.issubdtype(X.dtype, np.floating):
        X = X.astype(np.float64)
    e, c, nb = engine.bin_edges(X, int(d["n_bins"]))
    _assert_edges(e, c, nb, d["edges"], d["counts"], d["nan_bin_id"], name)
    ids = engine.bin_features(X, e, c, nb)
    assert hashlib.sha256(ids.tobytes()).hexdigest() == str(d["X_bin_sha"])


def _stress(seed, n=6000):
    rng = np.random.default_rng(seed)
    nan = lambda a, f: np.where(rng.random(n) < f, np.nan, a)
    cols = [
        rng.standard_normal(n),
        rng.integers(0, 7, n).astype(np.float64),
        nan(rng.exponential(size=n), 0.3),
        np.full(n, 3.25),
        np.full(n, np.nan),
        rng.choice([-0.0, 0.0, 1.0, -1.0], n),
        rng.random(n) * 1e-9,
        nan(rng.random(n) * 1e-9, 0.1),
        np.round(rng.standard_normal(n), 1),
        rng.integers(0, 300, n).astype(np.float64),
        np.concatenate([np.zeros(n - 40), rng.standard_normal(40)]),
        rng.standard_normal(n) * 1e30,
        np.where(rng.random(n) < 0.02, np.inf, rng.standard_normal(n)),
        np.where(rng.random(n) < 0.02, -np.inf, nan(rng.standard_normal(n), 0.05)),
        nan(rng.integers(0, 255, n).astype(np.float64), 0.2),
        nan(rng.integers(0, 254, n).astype(np.float64), 0.2),
        rng.standard_normal(n).astype(np.float32).astype(np.float64) * 7.0,
    ]
    return np.stack(cols, axis=1)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("n_bins", [255, 64, 2])
def test_edges_and_ids_match_host_on_edge_cases(engine, dtype, n_bins):
    from bsscl_gbm_b200 import binning
    X = _stress(11).astype(dtype)
    with np.errstate(invalid="ignore"):
        want = binning.build_bin_edges(X, n_bins)
    e, c, nb = engine.bin_edges(X, n_bins)
    _assert_edges(e, c, nb, *want, f"{np.dtype(dtype).name} n_bins={n_bins}")
    ids = engine.bin_features(X, e, c, nb)
    _assert_ids(ids, binning.bin_features(X, *want), X, e, c, "training rows")
    # rows at predict time: NaN in features that had none, values outside the range
    Xp = _stress(12).astype(dtype)
    Xp[::7, 0] = np.nan
    Xp[::5, 1] = 1e6
    Xp[::3, 3] = -1e6
    _assert_ids(engine.bin_features(Xp, e, c, nb), binning.bin_features(Xp, *want), Xp, e, c,
                "predict rows")


def test_edges_categorical_rows(engine):
    from bsscl_gbm_b200 import binning
    X = _stress(3)[:, :6]
    e, c, nb = engine.bin_edges(X, 255, categorical=[2, 4])
    want = binning.build_bin_edges(X, 255, categorical_features=[2, 4])
    _assert_edges(e, c, nb, *want, "categorical")


def test_edges_at_scale_match_host(engine):
    """1M rows: multi-chunk uploads, long radix sorts, scans that stop early."""
    from bsscl_gbm_b200 import datasets as D, binning
    X, _ = D.config4(n=1_000_000)
    X = np.ascontiguousarray(X[:, ::4])   # 25 of the 100 columns: normal, exponential, integer levels
    want = binning.build_bin_edges(X, 255)
    e, c, nb = engine.bin_edges(X, 255)
    _assert_edges(e, c, nb, *want, "config4 1M")
    ids = engine.bin_features(X[:200_000], e, c, nb)
    assert np.array_equal(ids, binning.bin_features(X[:200_000], *want))


def test_predict_raw_equals_predict_binned(engine):
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M, binning
    X, y, Xte = fit_inputs("cfg4_small")
    m = M(n_estimators=6, max_depth=6, n_bins=255, random_state=1, verbose=False).fit(X, y)
    p_raw = m.predict_proba(Xte)
    Xb = binning.bin_features(Xte, m.bin_edges, m.feature_bin_counts, m._nan_bin_id)
    assert np.array_equal(p_raw, m.predict_proba_binned(Xb))


def test_fit_on_device_bins_equals_fit_on_host_bins():
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M, binning
    X, y, _ = fit_inputs("cfg3_small")
    kw = dict(n_estimators=10, max_depth=6, class_weight="balanced_sqrt", n_bins=255,
              random_state=4, verbose=False)
    a = M(**kw).fit(X, y)                                   # edges and bins on the GPU
    e, c, nb = binning.build_bin_edges(X, 255)               # edges and bins on the host
    Xb = binning.bin_features(X, e, c, nb)
    b = M(**kw)
    for k in ("n_estimators", "max_depth", "learning_rate", "min_child_weight", "subsample",
              "colsample_bytree", "max_leaves", "reg_lambda", "gamma", "min_samples_leaf"):
        setattr(b, k, getattr(a, k))                            # the resolved hyper-parameters
    b.fit_binned(Xb, y, c)
    assert len(a.trees) == len(b.trees)
    for ta, tb in zip(a.trees, b.trees):
        nc = ta[5]
        assert nc == tb[5]
        for i in (0, 1, 2, 3, 4, 6):
            assert np.array_equal(np.asarray(ta[i])[:nc], np.asarray(tb[i])[:nc])
