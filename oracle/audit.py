"""Tie audit: explain a topology difference between two tree builders.

TEST INFRASTRUCTURE ONLY.

The reference sums float64 gradients in row order (E:582-596) and so breaks
mathematically equal gains by rounding noise; the engine sums them exactly.
Where their trees differ, ``audit_first_divergence`` finds the first node
whose split differs, takes that node's in-bag rows, and evaluates both
candidate splits with the reference's gain formula (E:614-617) in exact
rational arithmetic (every float64 g/h is an exact dyadic rational).  A
difference is "explained" when the two exact gains are equal (an exact tie)
or within ``rel_tol`` (a near tie below float64 resolution of the sums).
"""

from __future__ import annotations

from fractions import Fraction

import numpy as np


def _exact_ints(x):
    """float64 array -> (python ints m_i, common exponent E) with x_i = m_i * 2^-E."""
    E = 1100
    out = []
    for v in x.tolist():
        num, den = float(v).as_integer_ratio()
        out.append(num * ((1 << E) // den))
    return out, E


def node_rows(tree, X_bin, sample_idx, node):
    """In-bag rows reaching `node` of a (tf, tt, tv, tl, tr, nc, sg) tree."""
    tf, tt, _, tl, tr, nc, _ = tree
    parent = {}
    for k in range(nc):
        if tf[k] >= 0:
            parent[int(tl[k])] = (k, True)
            parent[int(tr[k])] = (k, False)
    mask = np.ones(len(sample_idx), dtype=bool)
    c = node
    while c in parent:
        p_, left = parent[c]
        go = X_bin[sample_idx, tf[p_]].astype(np.int64) <= tt[p_]
        mask &= go if left else ~go
        c = p_
    return np.asarray(sample_idx)[mask]


def exact_gain(X_bin, g, h, rows, counts, feat, thr, lam, mcw):
    """Exact gain of splitting `rows` on bin(feat) <= thr, or None if HL/HR < mcw."""
    gi, E = _exact_ints(g[rows])
    hi, _ = _exact_ints(h[rows])
    nb = int(counts[feat])
    b = np.minimum(X_bin[rows, feat].astype(np.int64), nb - 1)
    GL = sum(v for v, bb in zip(gi, b) if bb <= thr)
    HL = sum(v for v, bb in zip(hi, b) if bb <= thr)
    G, H = sum(gi), sum(hi)
    sc = Fraction(1, 1 << E)
    GL, HL, G, H = GL * sc, HL * sc, G * sc, H * sc
    GR, HR = G - GL, H - HL
    lam, mcw = Fraction(lam), Fraction(mcw)
    if HL < mcw or HR < mcw:
        return None
    return GL * GL / (HL + lam) + GR * GR / (HR + lam) - G * G / (H + lam)


def first_divergence(trees_a, trees_b):
    """(tree index, node id) of the first differing split, or None."""
    for t, (a, b) in enumerate(zip(trees_a, trees_b)):
        na, nb_ = a[5], b[5]
        for k in range(min(na, nb_)):
            if a[0][k] != b[0][k] or a[1][k] != b[1][k] or a[3][k] != b[3][k] or a[4][k] != b[4][k]:
                return t, k
        if na != nb_:
            return t, min(na, nb_)
    return None


def audit_node(X_bin, g, h, sample_idx, counts, tree_a, tree_b, node, lam, mcw):
    """Compare the two trees' splits at `node` exactly.  Returns a dict."""
    fa, ta = int(tree_a[0][node]), int(tree_a[1][node])
    fb, tb = int(tree_b[0][node]), int(tree_b[1][node])
    out = {"node": node, "a": (fa, ta), "b": (fb, tb)}
    if fa < 0 or fb < 0:
        out["kind"] = "structural"
        return out
    rows = node_rows(tree_a, X_bin, sample_idx, node)
    rows_b = node_rows(tree_b, X_bin, sample_idx, node)
    if len(rows) != len(rows_b) or not np.array_equal(np.sort(rows), np.sort(rows_b)):
        out["kind"] = "structural"
        return out
    # same partition (e.g. neighbouring empty bins): identical children
    ga = X_bin[rows, fa].astype(np.int64) <= ta
    gb = X_bin[rows, fb].astype(np.int64) <= tb
    if np.array_equal(ga, gb):
        out["kind"] = "same_partition"
        return out
    A = exact_gain(X_bin, g, h, rows, counts, fa, ta, lam, mcw)
    B = exact_gain(X_bin, g, h, rows, counts, fb, tb, lam, mcw)
    out["gain_a"], out["gain_b"] = A, B
    if A is None or B is None:
        out["kind"] = "mcw_boundary"
    elif A == B:
        out["kind"] = "exact_tie"
    else:
        out["kind"] = "near_tie"
        out["rel_gap"] = float(abs(A - B) / max(abs(A), abs(B)))
    out["n_rows"] = int(len(rows))
    return out


def explained(res, rel_tol=1e-9):
    k = res.get("kind")
    if k in ("exact_tie", "same_partition"):
        return True
    if k == "near_tie":
        return res["rel_gap"] < rel_tol
    return False
