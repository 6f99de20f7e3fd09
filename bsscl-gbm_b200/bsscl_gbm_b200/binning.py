"""Bin edges and binning, restated from the reference on the host.

``build_bin_edges`` follows ``_build_bin_edges``
(src/bsscl_gbm/estimator_v1_0_1.py:2073-2141): per feature, NaN gets its own
bin 0 and shifts the numeric bins by one; up to ``n_bins`` (minus one with a
NaN bin) numeric bins come from the sorted unique values, or from
``np.percentile`` at ``linspace(0, 1, k)`` when there are more uniques; an
edge ``e[-1] + 1e-8`` is appended (a no-op in float32, where NumPy keeps the
scalar in float32 -- the reason the column maximum can land one id past the
last bin); rows are padded with the last edge into ``edges_2d[p, max_b]``.

``bin_features`` gives the ids of ``_bin_features`` (E:2144-2189) with the
'standard' search of E:204-226 (the 'hybrid' search of E:155-202 returns
the same id for every non-NaN value): the largest ``k`` with
``edges[k] <= v`` after the early outs ``v < edges[0] -> 0`` and
``v >= edges[nb] -> nb - 1``.  NaN is read as 0.0 when any training feature
had a NaN (E:2157-2162), otherwise it falls to bin 0 of the search.
"""

from __future__ import annotations

import numpy as np


def build_bin_edges(X, n_bins, categorical_features=None, sample_weight=None):
    """Returns ``(edges_2d float64 [p, max_b], bin_counts int32 [p], nan_bin_id int32 [p])``."""
    p = X.shape[1]
    counts = np.zeros(p, dtype=np.int32)
    nan_bin = np.full(p, -1, dtype=np.int32)
    per_feature = []
    cat = set(categorical_features) if categorical_features is not None else set()
    for j in range(p):
        if j in cat:
            per_feature.append(np.arange(-0.5, 64.5, 1.0))
            counts[j] = 64
            continue
        col = X[:, j]
        nan_mask = np.isnan(col)
        has_nan = bool(np.any(nan_mask))
        if has_nan:
            nan_bin[j] = 0
            clean = col[~nan_mask]
            if clean.size == 0:
                per_feature.append(np.array([0.0, 1.0]))
                counts[j] = 1
                continue
        else:
            clean = col
        uniq = np.unique(clean)
        numeric_bins = n_bins - (1 if has_nan else 0)
        if len(uniq) <= numeric_bins:
            e = np.sort(uniq)
        else:
            q = np.linspace(0, 1, min(numeric_bins + 1, len(uniq)))
            if sample_weight is not None:
                sw = sample_weight[~nan_mask] if has_nan else sample_weight
                order = np.argsort(clean)
                cs, ws = clean[order], sw[order]
                cw = np.cumsum(ws) - 0.5 * ws
                cw /= np.sum(ws)
                e = np.unique(np.interp(q, cw, cs))
            else:
                e = np.unique(np.percentile(clean, q * 100))
        e = np.append(e, e[-1] + 1e-8)
        per_feature.append(e)
        counts[j] = len(e) if has_nan else len(e) - 1
    max_b = int(np.max(counts)) + 1
    edges = np.zeros((p, max_b), dtype=np.float64)
    for j, e in enumerate(per_feature):
        edges[j, :len(e)] = e
        edges[j, len(e):] = e[-1]
    return edges, counts, nan_bin


def bin_features(X, edges, counts, nan_bin_id):
    """Raw bin ids (uint16 [n, p]) exactly as the reference's ``_bin_features``."""
    n, p = X.shape
    has_any_nan = nan_bin_id is not None and bool(np.any(nan_bin_id >= 0))
    out = np.empty((n, p), dtype=np.uint16)
    for j in range(p):
        v = np.asarray(X[:, j], dtype=np.float64)
        isn = np.isnan(v)
        if has_any_nan:
            v = np.where(isn, 0.0, v)
        nb = int(counts[j])
        e = edges[j]
        b = np.searchsorted(e[:nb], v, side="right") - 1
        np.clip(b, 0, nb - 1, out=b)
        b[v >= e[nb]] = nb - 1
        if not has_any_nan:
            b[isn] = 0
        if has_any_nan and nan_bin_id[j] >= 0:
            b = np.where(isn, 0, b + 1)
        out[:, j] = b
    return out


def device_bins(X_bin, counts):
    """Ids for the device: ``min(id, bin_count - 1)``, as uint8 -- or as
    uint16 when a feature has 257 bins (n_bins 256 with a NaN bin,
    E:2111-2127), whose id 256 the device keeps as a row bit.

    Lossless for training and predict: the histogram clamps ids >= bin_count
    the same way (E:593-594), and no threshold exceeds bin_count - 2
    (E:604), so the clamped id always goes right whenever the raw one did.
    """
    lim = np.asarray(counts, dtype=np.int64) - 1
    if int(lim.max()) > 256:
        raise ValueError("the device path holds at most 257 bins per feature "
                         f"(feature with {int(lim.max()) + 1} bins); use n_bins <= 256")
    X_bin = np.asarray(X_bin)
    if int(lim.max()) == 256:
        return np.minimum(X_bin, lim[None, :].astype(X_bin.dtype)).astype(np.uint16)
    return np.minimum(X_bin, lim[None, :].astype(X_bin.dtype)).astype(np.uint8)
