"""Seeded synthetic stand-ins for the reference's benchmark workloads.

The reference quotes its numbers on public datasets (credit-card fraud, a
noisy-label set, a Higgs subset) and on ``make_classification`` matrices.
None of those records are reproduced here: every generator below draws
seeded synthetic data with the shapes, sizes and value distributions of the
five benchmark configurations (1: 12k x 30 f64; 2: 284,807 x 30 f64 with
0.17 % positives; 3: 50k x 20 noisy two-cluster data; 4: 1M x 100 f32 with
30 % NaN; 5: 10M x 200 pre-binned uint8).
"""

from __future__ import annotations

import numpy as np


def _sigmoid(z):
    return 1.0 / (1.0 + np.exp(-z))


def _solve_intercept(logit, rate, iters=200):
    """Bisection for ``b`` with ``mean(sigmoid(logit + b)) == rate``."""
    lo, hi = -60.0, 60.0
    for _ in range(iters):
        mid = 0.5 * (lo + hi)
        if _sigmoid(logit + mid).mean() > rate:
            hi = mid
        else:
            lo = mid
    return 0.5 * (lo + hi)


def config1(n_train=10_000, n_test=2_000, p=30, seed=0, positive_rate=0.37):
    """Config 1: N(0,1) f64 features, label ~ Bernoulli(sigmoid(x.w + 0.5 x0 x1 + b)).

    ``b`` is solved on the training rows so that the expected positive rate is
    ``positive_rate`` (the plain recipe gives ~50 %; the benchmark text asks
    for ~37 %).  Returns ``(X_train, y_train, X_test, y_test)``.
    """
    rng = np.random.default_rng(seed)
    n = n_train + n_test
    X = rng.standard_normal((n, p))
    w = rng.standard_normal(p)
    logit = X @ w + 0.5 * X[:, 0] * X[:, 1]
    b = _solve_intercept(logit[:n_train], positive_rate)
    y = (rng.random(n) < _sigmoid(logit + b)).astype(np.int64)
    return X[:n_train], y[:n_train], X[n_train:], y[n_train:]


def config2(n=284_807, seed=1, n_pos=492):
    """Config 2: extreme imbalance, 30 f64 columns.

    Columns 0-27 ~ N(0, s_j^2) with s_j = linspace(2.0, 0.3, 28); column 28 ~
    U(0, 172800) (a time stamp); column 29 ~ LogNormal(3, 1.5) (an amount).
    ``n_pos`` rows chosen without replacement are positive and get +1.5 s_j
    on 10 randomly chosen Gaussian columns.
    """
    rng = np.random.default_rng(seed)
    sig = np.linspace(2.0, 0.3, 28)
    X = np.empty((n, 30), dtype=np.float64)
    X[:, :28] = rng.standard_normal((n, 28)) * sig
    X[:, 28] = rng.uniform(0.0, 172_800.0, n)
    X[:, 29] = rng.lognormal(3.0, 1.5, n)
    pos = rng.choice(n, size=n_pos, replace=False)
    cols = rng.choice(28, size=10, replace=False)
    y = np.zeros(n, dtype=np.int64)
    y[pos] = 1
    for c in cols:
        X[pos, c] += 1.5 * sig[c]
    return X, y


def config3(n=50_000, p=20, seed=2, minority=0.02, flip=0.05, sep=0.6):
    """Config 3: two unit-covariance Gaussian clusters ``sep`` apart, 98/2, 5 % flips."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal(p)
    u /= np.linalg.norm(u)
    y = (rng.random(n) < minority).astype(np.int64)
    X = rng.standard_normal((n, p)) + np.outer(y * sep, u)
    flips = rng.random(n) < flip
    y = np.where(flips, 1 - y, y)
    return X, y


def config4(n=1_000_000, seed=3, nan_frac=0.30, positive_rate=0.01):
    """Config 4: 1M x 100 float32, 30 % NaN everywhere, 99/1 sparse-logistic label.

    60 N(0,1) columns, 30 Exp(1) columns and 10 integer-valued columns with
    2-50 levels each (plain numeric columns, no categorical encoding).  The
    label comes from a logistic model on 15 random features (NaN read as 0)
    with an intercept solved for a 1 % positive rate.
    """
    rng = np.random.default_rng(seed)
    X = np.empty((n, 100), dtype=np.float32)
    X[:, :60] = rng.standard_normal((n, 60), dtype=np.float32)
    X[:, 60:90] = rng.exponential(1.0, (n, 30)).astype(np.float32)
    levels = rng.integers(2, 51, size=10)
    for k in range(10):
        X[:, 90 + k] = rng.integers(0, levels[k], size=n).astype(np.float32)
    feats = rng.choice(100, size=15, replace=False)
    wts = rng.standard_normal(15)
    logit = X[:, feats].astype(np.float64) @ wts
    b = _solve_intercept(logit, positive_rate)
    y = (rng.random(n) < _sigmoid(logit + b)).astype(np.int64)
    mask = rng.random((n, 100), dtype=np.float32) < nan_frac
    X[mask] = np.nan
    return X, y


def config5_bins(n=10_000_000, p=200, seed=5, nan_frac=0.10, positive_rate=0.05, rows=None):
    """Config 5: pre-binned uint8 matrix ~ U{1..254} with 10 % NaN-bin (0) entries.

    Returns ``(X_bin uint8 [m, p] row-major, y int64 [n])`` where X_bin holds
    rows ``rows = (lo, hi)`` (default: all n) and y is always every row's
    label.  Rows are made in blocks of 2^20 from their own seeds, so any row
    range is the same data whichever process makes it.  Every feature
    carries a NaN bin, so each has 256 bin ids (0 = NaN, 1..255 numeric).
    """
    lo, hi = rows if rows is not None else (0, n)
    blk = 1 << 20
    Xb = np.empty((hi - lo, p), dtype=np.uint8)
    for b0 in range((lo // blk) * blk, hi, blk):
        r = np.random.default_rng([seed, b0 // blk])
        m = min(blk, n - b0)
        xb = r.integers(1, 255, size=(m, p), dtype=np.uint8)
        xb[r.random((m, p), dtype=np.float32) < nan_frac] = 0
        a, z = max(lo, b0), min(hi, b0 + m)
        Xb[a - lo:z - lo] = xb[a - b0:z - b0]
    y = (np.random.default_rng([seed, 1 << 30]).random(n) < positive_rate).astype(np.int64)
    return Xb, y


def config5_ensemble(n_trees=1000, depth=8, p=200, seed=5, max_threshold=253):
    """Config 5 predict ensemble: ``n_trees`` full depth-``depth`` trees of random splits.

    Packed exactly like the reference's ``_pack_tree_list`` output: features
    int16 (-1 for leaves), thresholds int64, values float64, left/right int32
    (tree-local ids), offsets int32[T+1].  Internal node ``k`` has children
    ``2k+1`` and ``2k+2`` (BFS numbering); leaf values ~ N(0, 0.1).
    """
    rng = np.random.default_rng(seed)
    nodes = (1 << (depth + 1)) - 1
    n_int = (1 << depth) - 1
    feat = np.full((n_trees, nodes), -1, dtype=np.int16)
    thr = np.zeros((n_trees, nodes), dtype=np.int64)
    val = np.zeros((n_trees, nodes), dtype=np.float64)
    left = np.full((n_trees, nodes), -1, dtype=np.int32)
    right = np.full((n_trees, nodes), -1, dtype=np.int32)
    feat[:, :n_int] = rng.integers(0, p, size=(n_trees, n_int))
    thr[:, :n_int] = rng.integers(0, max_threshold + 1, size=(n_trees, n_int))
    val[:, :] = rng.normal(0.0, 0.1, size=(n_trees, nodes))
    k = np.arange(n_int, dtype=np.int32)
    left[:, :n_int] = 2 * k + 1
    right[:, :n_int] = 2 * k + 2
    offsets = (np.arange(n_trees + 1, dtype=np.int64) * nodes).astype(np.int32)
    return {
        "features": feat.reshape(-1), "thresholds": thr.reshape(-1),
        "values": val.reshape(-1), "left": left.reshape(-1),
        "right": right.reshape(-1), "offsets": offsets,
    }


def multiclass(n=8_000, p=12, K=4, seed=7, nan_frac=0.05):
    """A K-class stand-in for the reference's multi-class path (E:2949-3065):
    Gaussian class clusters in p dimensions with unequal class sizes (class k
    has weight proportional to 1 / (k + 1)), NaN in the last three columns."""
    rng = np.random.default_rng(seed)
    pri = 1.0 / np.arange(1, K + 1)
    y = rng.choice(K, size=n, p=pri / pri.sum())
    centres = rng.standard_normal((K, p)) * 1.2
    X = centres[y] + rng.standard_normal((n, p))
    X[:, -3:][rng.random((n, 3)) < nan_frac] = np.nan
    return X, y.astype(np.int64)


def regression(n=8_000, p=10, seed=9, nan_frac=0.05, scale=100.0):
    """A stand-in for the reference's regression path (E:2607-2705): targets
    ``scale * (sin(x0) + x1 * x2 / 2 + 0.3 x3^2) + N(0, scale / 10)``, NaN in
    the last two columns."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, p))
    y = scale * (np.sin(X[:, 0]) + 0.5 * X[:, 1] * X[:, 2] + 0.3 * X[:, 3] ** 2) \
        + rng.standard_normal(n) * (scale / 10.0)
    X[:, -2:][rng.random((n, 2)) < nan_frac] = np.nan
    return X, y


def top_bin(n=20_000, p=30, seed=21, nan_frac=0.2, n_top=60):
    """Data for the reference's default constructor (``n_bins='auto'``:
    256 bins once p >= 28, E:2111-2127), where every continuous feature gets
    257 bin ids.  N(0,1) float64 features, ``nan_frac`` NaN in the first
    ten; in features 3 (with NaN) and 12 (without) ``n_top`` rows -- fewer
    than 1/256 of the rows, so the quantile edges stay distinct -- are set
    to the column maximum and labelled positive, so that a threshold of 255
    (bin 256 alone on the right) is worth a split.
    """
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, p))
    logit = 1.2 * X[:, 0] - 0.8 * X[:, 5] + 0.6 * X[:, 12] * X[:, 7]
    y = (rng.random(n) < _sigmoid(logit + _solve_intercept(logit, 0.15))).astype(np.int64)
    X[:, :10][rng.random((n, 10)) < nan_frac] = np.nan
    for j in (3, 12):
        col = X[:, j]
        finite = np.flatnonzero(~np.isnan(col))
        top = rng.choice(finite, size=n_top, replace=False)
        col[top] = np.nanmax(col)
        y[top] = 1
    return X, y
