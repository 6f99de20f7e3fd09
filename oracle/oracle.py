"""ctypes bindings and a boosting driver for the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU legs as the checker.  The product package never imports it.

``fit_binary`` restates the reference's binary boosting loop
(src/bsscl_gbm/estimator_v1_0_1.py, ``_fit_binary`` E:2825-2944) around the
C builders: class weights (E:2570-2603), weighted-mean base score
(E:2829-2835), p = sigmoid(clip(F)) / g / h (E:2861, E:2873-2874), the
cumulative ``RandomState.shuffle`` sampler (E:2502-2517, using NumPy's own
legacy generator), tree build + post-prune (E:2397-2459), the monotone
clip (E:2461-2499), the F update ``F += lr * tree(X)`` (E:2896-2897) and the
train logloss (E:2905).  ``scale_pos_weight`` with ``objective='binary'``
sets the class weights (E:2572-2577).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

MODE_REF = 0
MODE_EXACT = 1

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        i32, i64, f64 = C.c_int32, C.c_int64, C.c_double
        L.or_bin_matrix.argtypes = [P, i64, i32, P, i32, P, P, i32, i32, P]
        L.or_build_leafwise.argtypes = [P, i64, i32, P, P, P, i64, P, i32, P, i32, i32, i32,
                                        i32, f64, f64, f64, i32, i32, P, P, P, P, P, P, P]
        L.or_build_depthwise.argtypes = [P, i64, i32, P, P, P, i64, P, i32, P, i32, i32, i32,
                                         f64, f64, f64, i32, i32, P, P, P, P, P, P, P]
        L.or_post_prune.argtypes = [P, P, P, P, f64, i32]
        L.or_leaf_ids.argtypes = [P, i64, i32, P, P, P, P, P]
        L.or_predict_packed.argtypes = [P, i64, i32, P, P, P, P, P, P, i32, f64, P, P]
        L.or_set_nan_dir.argtypes = [P]
        L.or_set_nan_dir.restype = None
        L.or_grad_hess.argtypes = [P, P, P, i64, P, P]
        L.or_logloss.argtypes = [P, P, i64]
        L.or_logloss.restype = C.c_double
        L.or_num_threads.restype = C.c_int
        L.or_i128_to_double.argtypes = [C.c_int64, C.c_uint64]
        L.or_i128_to_double.restype = C.c_double
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def i128_to_double(v):
    """The oracle's conversion of a Python int in [-2^127, 2^127) to float64."""
    hi = v >> 64
    lo = v & ((1 << 64) - 1)
    return lib().or_i128_to_double(hi, lo)


def num_threads():
    return lib().or_num_threads()


def bin_matrix(X, edges, counts, nan_bin_id, hybrid):
    X = np.ascontiguousarray(X, dtype=np.float64)
    n, p = X.shape
    edges = np.ascontiguousarray(edges, dtype=np.float64)
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    nan_bin_id = np.ascontiguousarray(nan_bin_id, dtype=np.int32)
    out = np.empty((n, p), dtype=np.uint16)
    has_any = int(np.any(nan_bin_id >= 0))
    lib().or_bin_matrix(_p(X), n, p, _p(edges), edges.shape[1], _p(counts), _p(nan_bin_id),
                        has_any, int(bool(hybrid)), _p(out))
    return out


def build_tree(X_bin, g, h, sample_idx, feat_idx, counts, *, max_leaves=63, max_depth=6,
               msl=5, mcw=1.0, lam=1.0, gamma=0.0, mode=MODE_REF, scale_bits=0,
               policy="leaf", nan_bin_id=None):
    """One tree.  Returns ``(tf, tt, tv, tl, tr, nc, sg)`` like the reference.

    ``nan_bin_id`` (the reference's ``_nan_bin_id``, 0 where bin 0 is a NaN
    bin): also evaluate the splits that send NaN right (the engine's
    ``nan_direction``); the tree's ``tt`` then carries the direction in bit
    32 (``split_nan_right`` separates them)."""
    Xb = np.ascontiguousarray(X_bin, dtype=np.uint16)
    n, p = Xb.shape
    g = np.ascontiguousarray(g, dtype=np.float64)
    h = np.ascontiguousarray(h, dtype=np.float64)
    sidx = np.ascontiguousarray(sample_idx, dtype=np.int64)
    fidx = np.ascontiguousarray(feat_idx, dtype=np.int32)
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    max_bins = int(counts.max())
    if policy == "leaf":
        M = 2 * max_leaves + 2
    else:
        M = (1 << (max_depth + 1)) - 1
    tf = np.empty(M, np.int32); tt = np.empty(M, np.int64); tv = np.empty(M, np.float64)
    tl = np.empty(M, np.int32); tr = np.empty(M, np.int32); sg = np.empty(M, np.float64)
    nc = C.c_int32(0)
    nanf = None if nan_bin_id is None else (np.asarray(nan_bin_id) == 0).astype(np.uint8)
    lib().or_set_nan_dir(_p(nanf))
    if policy == "leaf":
        rc = lib().or_build_leafwise(_p(Xb), n, p, _p(g), _p(h), _p(sidx), len(sidx), _p(fidx),
                                     len(fidx), _p(counts), max_bins, max_leaves, max_depth,
                                     msl, mcw, lam, gamma, mode, scale_bits, _p(tf), _p(tt),
                                     _p(tv), _p(tl), _p(tr), _p(sg), C.byref(nc))
    else:
        rc = lib().or_build_depthwise(_p(Xb), n, p, _p(g), _p(h), _p(sidx), len(sidx),
                                      _p(fidx), len(fidx), _p(counts), max_bins, max_depth,
                                      msl, mcw, lam, gamma, mode, scale_bits, _p(tf), _p(tt),
                                      _p(tv), _p(tl), _p(tr), _p(sg), C.byref(nc))
    lib().or_set_nan_dir(None)
    if rc != 0:
        raise MemoryError("oracle builder failed to allocate")
    return tf, tt, tv, tl, tr, int(nc.value), sg


def split_nan_right(tt):
    """(thresholds, nan_right) of a tree built with nan_bin_id."""
    tt = np.asarray(tt, np.int64)
    return tt & 0xFFFFFFFF, (tt >> 32).astype(np.int32)


def post_prune(tf, tl, tr, sg, gamma, nc):
    lib().or_post_prune(_p(tf), _p(tl), _p(tr), _p(sg), float(gamma), int(nc))


def enforce_monotone(tf, tl, tr, tv, nc, mono):
    """The reference's post-hoc monotone clip (E:2461-2499), in place on tv:
    nodes in index order; a split on a feature with constraint +1 (-1) whose
    left child value is above (below) the right's sets both children to
    (left + right) / 2.  Nodes past a pruned split are visited as well, as in
    the reference's loop over range(nc)."""
    if mono is None:
        return
    for k in range(int(nc)):
        f = int(tf[k])
        if f < 0:
            continue
        c = int(mono[f])
        if c == 0:
            continue
        l, r = int(tl[k]), int(tr[k])
        if l < 0 or r < 0:
            continue
        lv, rv = float(tv[l]), float(tv[r])
        if (c == 1 and lv > rv) or (c == -1 and lv < rv):
            m = (lv + rv) / 2.0
            tv[l] = m
            tv[r] = m


def leaf_ids(X_bin, tf, tt, tl, tr, nan_right=None):
    """Leaf id of every row; ``nan_right`` [nodes] (or bit 32 of ``tt``) sends NaN right."""
    if nan_right is not None:
        tt = np.asarray(tt, np.int64) | (np.asarray(nan_right, np.int64) << 32)
    Xb = np.ascontiguousarray(X_bin, dtype=np.uint16)
    n, p = Xb.shape
    out = np.empty(n, np.int32)
    lib().or_leaf_ids(_p(Xb), n, p, _p(np.ascontiguousarray(tf, np.int32)),
                      _p(np.ascontiguousarray(tt, np.int64)), _p(np.ascontiguousarray(tl, np.int32)),
                      _p(np.ascontiguousarray(tr, np.int32)), _p(out))
    return out


def predict_packed(X_bin, packed, n_trees, lr):
    Xb = np.ascontiguousarray(X_bin, dtype=np.uint16)
    n, p = Xb.shape
    F = np.empty(n, np.float64)
    a = {k: np.ascontiguousarray(v) for k, v in packed.items() if v is not None}
    nr = a.get("nan_right")
    lib().or_predict_packed(_p(Xb), n, p, _p(a["features"].astype(np.int16)),
                            _p(a["thresholds"].astype(np.int64)), _p(a["values"].astype(np.float64)),
                            _p(a["left"].astype(np.int32)), _p(a["right"].astype(np.int32)),
                            _p(a["offsets"].astype(np.int32)), int(n_trees), float(lr),
                            _p(None if nr is None else nr.astype(np.uint8)), _p(F))
    return F


def grad_hess(F, y01, w2):
    F = np.ascontiguousarray(F, np.float64)
    y = np.ascontiguousarray(y01, np.uint8)
    w2 = np.ascontiguousarray(w2, np.float64)
    g = np.empty_like(F); h = np.empty_like(F)
    lib().or_grad_hess(_p(F), _p(y), _p(w2), len(F), _p(g), _p(h))
    return g, h


def grad_hess_numpy(F, y01, w2):
    """The reference's binary gradients in NumPy's own arithmetic
    (E:2859-2868: p = 1 / (1 + np.exp(-clip(F, -500, 500))), g = w (p - y),
    h = w p (1 - p)).  NumPy's vectorised exp can differ from the C
    library's in the last bit, so MODE_REF uses this one to stay bit-exact
    with the reference."""
    y = np.asarray(y01).astype(np.int64)
    sw = np.asarray(w2, np.float64)[y]
    p = 1.0 / (1.0 + np.exp(-np.clip(np.asarray(F, np.float64), -500, 500)))
    return sw * (p - y), sw * p * (1.0 - p)


def logloss(F, y01):
    F = np.ascontiguousarray(F, np.float64)
    y = np.ascontiguousarray(y01, np.uint8)
    return lib().or_logloss(_p(F), _p(y), len(F))


# ----------------------------------------------------------------------------
# Boosting driver
# ----------------------------------------------------------------------------

def class_weights(y01, class_weight, scale_pos_weight=None, objective="auto"):
    """Per-class weights ``w[2]`` (E:2570-2603).  ``scale_pos_weight`` only acts
    when ``objective == 'binary'`` (E:2572)."""
    n = len(y01)
    if scale_pos_weight is not None and objective == "binary":
        return np.array([1.0, float(scale_pos_weight)])
    if class_weight not in ("balanced", "balanced_sqrt"):
        return np.array([1.0, 1.0])
    w = np.ones(2)
    for k in range(2):
        nk = int(np.sum(y01 == k))
        wk = n / (2 * max(nk, 1))
        if class_weight == "balanced_sqrt":
            wk = wk ** 0.35
        w[k] = wk
    return w


def base_score(y01, w2):
    sw = w2[y01]
    p0 = np.clip(np.average(y01, weights=sw), 1e-7, 1.0 - 1e-7)
    return float(np.log(p0 / (1.0 - p0)))


def fit_binary(X_bin, y01, counts, *, n_estimators, learning_rate, max_leaves, max_depth,
               min_samples_leaf, min_child_weight, reg_lambda, gamma, subsample,
               colsample, class_weight, random_state, mode=MODE_REF, scale_bits=None,
               grow_policy="leaf", record=None, monotone=None, scale_pos_weight=None, objective="auto"):
    """The reference's ``_fit_binary`` loop on the oracle builders.

    ``scale_bits=None`` in MODE_EXACT picks S per round the way the engine
    does (``engine_scale_bits``).  ``monotone``: int32 [p] of -1/0/+1, the
    reference's ``_mono_arr``.  Returns a dict with trees, base score, final
    F and the train-loss history.
    """
    y01 = np.asarray(y01).astype(np.int64)
    n, p = X_bin.shape
    w2 = class_weights(y01, class_weight, scale_pos_weight, objective)
    base = base_score(y01, w2)
    F = np.full(n, base)
    n_sub = max(1, int(n * subsample))
    n_feat = max(1, int(p * colsample))
    rng = np.random.RandomState(random_state)
    all_r = np.arange(n, dtype=np.int64)
    all_f = np.arange(p, dtype=np.int32)
    trees, losses = [], []
    y8 = y01.astype(np.uint8)
    for m in range(n_estimators):
        g, h = grad_hess_numpy(F, y01, w2) if mode == MODE_REF else grad_hess(F, y8, w2)
        if subsample < 1.0:
            rng.shuffle(all_r)
            sidx = all_r[:n_sub].copy()
        else:
            sidx = all_r.copy()
        if colsample < 1.0:
            rng.shuffle(all_f)
            fidx = np.sort(all_f[:n_feat]).copy()
        else:
            fidx = all_f.copy()
        S = scale_bits
        if mode == MODE_EXACT and S is None:
            S = engine_scale_bits(len(sidx), w2)
        t = build_tree(X_bin, g, h, sidx, fidx, counts, max_leaves=max_leaves,
                       max_depth=max_depth, msl=min_samples_leaf, mcw=min_child_weight,
                       lam=reg_lambda, gamma=gamma, mode=mode, scale_bits=S or 0,
                       policy=grow_policy)
        tf, tt, tv, tl, tr, nc, sg = t
        post_prune(tf, tl, tr, sg, gamma, nc)          # E:2451-2452
        enforce_monotone(tf, tl, tr, tv, nc, monotone)  # E:2454-2457
        if record is not None:
            record.append(dict(g=g, h=h, sample=sidx, feat=fidx))
        leaf = leaf_ids(X_bin, tf, tt, tl, tr)
        F = F + learning_rate * tv[leaf]
        losses.append(logloss(F, y8))
        trees.append((tf, tt, tv, tl, tr, nc, sg))
    return dict(trees=trees, base_score=base, F=F, train_loss=np.array(losses), w2=w2)


def softmax(F):
    """``_softmax`` (E:2328-2332), NumPy's own arithmetic."""
    Fs = F - F.max(axis=1, keepdims=True)
    e = np.exp(Fs)
    return e / e.sum(axis=1, keepdims=True)


def mc_logloss(y_onehot, F):
    """``_compute_multiclass_logloss`` (E:2335-2341)."""
    proba = np.clip(softmax(F), 1e-15, 1 - 1e-15)
    return -np.mean(np.sum(y_onehot * np.log(proba), axis=1))


def class_weights_mc(y, K, class_weight):
    """Per-class weights ``w[K]`` of ``_compute_class_weights`` (E:2570-2603)
    for a K-class fit: ``n / (K max(n_k, 1))``, to the power 0.35 for
    'balanced_sqrt', ones otherwise."""
    y = np.asarray(y)
    n = len(y)
    w = np.ones(K, dtype=np.float64)
    if class_weight in ("balanced", "balanced_sqrt"):
        for k in range(K):
            n_k = np.sum(y == k)
            w_k = n / (K * max(n_k, 1))
            if class_weight == "balanced_sqrt":
                w_k = w_k ** 0.35
            w[k] = w_k
    return w


def fit_multiclass(X_bin, y, counts, K, *, n_estimators, learning_rate, max_leaves, max_depth,
                   min_samples_leaf, min_child_weight, reg_lambda, gamma, subsample, colsample,
                   class_weight, random_state, mode=MODE_REF, scale_bits=None, grow_policy="leaf",
                   record=None):
    """The reference's ``_fit_multiclass`` loop (E:2949-3065) on the oracle
    builders: per round one shared subsample, the softmax gradients of every
    class from the round's start, K trees, F of class k updated after its
    tree.  ``record`` gets per round (g [K][n], h [K][n], sample, feat)."""
    y = np.asarray(y).astype(np.int64)
    n, p = X_bin.shape
    y_onehot = np.eye(K, dtype=np.float64)[y]
    F = np.zeros((n, K), dtype=np.float64)
    w = class_weights_mc(y, K, class_weight)
    sw = w[y]
    n_sub = max(1, int(n * subsample))
    n_feat = max(1, int(p * colsample))
    rng = np.random.RandomState(random_state)
    all_r = np.arange(n, dtype=np.int64)
    all_f = np.arange(p, dtype=np.int32)
    trees = [[] for _ in range(K)]
    losses = []
    for m in range(n_estimators):
        proba = softmax(F)
        if subsample < 1.0:
            rng.shuffle(all_r)
            sidx = all_r[:n_sub].copy()
        else:
            sidx = all_r.copy()
        if colsample < 1.0:
            rng.shuffle(all_f)
            fidx = np.sort(all_f[:n_feat]).copy()
        else:
            fidx = all_f.copy()
        grad_all = sw[:, None] * (proba - y_onehot)
        hess_all = sw[:, None] * proba * (1.0 - proba)
        S = scale_bits
        if mode == MODE_EXACT and S is None:
            S = engine_scale_bits(len(sidx), w)
        gs, hs = [], []
        for k in range(K):
            g = np.ascontiguousarray(grad_all[:, k])
            h = np.maximum(np.ascontiguousarray(hess_all[:, k]), 1e-8)
            t = build_tree(X_bin, g, h, sidx, fidx, counts, max_leaves=max_leaves,
                           max_depth=max_depth, msl=min_samples_leaf, mcw=min_child_weight,
                           lam=reg_lambda, gamma=gamma, mode=mode, scale_bits=S or 0,
                           policy=grow_policy)
            tf, tt, tv, tl, tr, nc, sg = t
            post_prune(tf, tl, tr, sg, gamma, nc)
            leaf = leaf_ids(X_bin, tf, tt, tl, tr)
            F[:, k] += learning_rate * tv[leaf]
            trees[k].append((tf, tt, tv, tl, tr, nc, sg))
            gs.append(g)
            hs.append(h)
        if record is not None:
            record.append(dict(g=np.array(gs), h=np.array(hs), sample=sidx, feat=fidx))
        losses.append(mc_logloss(y_onehot, F))
    return dict(trees=trees, F=F, train_loss=np.array(losses), w=w)


def reg_scale_bits(gmax):
    """The engine's fixed-point exponent for a regression round:
    ``62 - ceil(log2(16384 * max(1, max|g|)))``."""
    return 62 - int(np.ceil(np.log2(16384.0 * max(1.0, float(gmax)))))


def fit_regression(X_bin, y, counts, *, n_estimators, learning_rate, max_leaves, max_depth,
                   min_samples_leaf, min_child_weight, reg_lambda, gamma, subsample, colsample,
                   random_state, loss="mse", mode=MODE_REF, grow_policy="leaf", record=None):
    """The reference's ``_fit_regression`` loop (E:2607-2705) on the oracle
    builders: F from mean(y), g = F - y (mse) or sign(F - y) (mae), h = 1.
    In MODE_EXACT each round's S follows its largest |g| as the engine's does."""
    y = np.asarray(y, dtype=np.float64)
    n, p = X_bin.shape
    init = float(np.mean(y))
    F = np.full(n, init, dtype=np.float64)
    n_sub = max(1, int(n * subsample))
    n_feat = max(1, int(p * colsample))
    rng = np.random.RandomState(random_state)
    all_r = np.arange(n, dtype=np.int64)
    all_f = np.arange(p, dtype=np.int32)
    trees, losses = [], []
    for m in range(n_estimators):
        g = F - y if loss == "mse" else np.sign(F - y)
        h = np.ones(n, dtype=np.float64)
        if subsample < 1.0:
            rng.shuffle(all_r)
            sidx = all_r[:n_sub].copy()
        else:
            sidx = all_r.copy()
        if colsample < 1.0:
            rng.shuffle(all_f)
            fidx = np.sort(all_f[:n_feat]).copy()
        else:
            fidx = all_f.copy()
        S = reg_scale_bits(1.0 if loss == "mae" else np.max(np.abs(g))) if mode == MODE_EXACT else 0
        t = build_tree(X_bin, g, h, sidx, fidx, counts, max_leaves=max_leaves, max_depth=max_depth,
                       msl=min_samples_leaf, mcw=min_child_weight, lam=reg_lambda, gamma=gamma, mode=mode,
                       scale_bits=S, policy=grow_policy)
        tf, tt, tv, tl, tr, nc, sg = t
        post_prune(tf, tl, tr, sg, gamma, nc)
        if record is not None:
            record.append(dict(g=g, h=h, sample=sidx, feat=fidx, S=S))
        leaf = leaf_ids(X_bin, tf, tt, tl, tr)
        F = F + learning_rate * tv[leaf]
        losses.append(np.mean((y - F) ** 2) if loss == "mse" else np.mean(np.abs(y - F)))
        trees.append((tf, tt, tv, tl, tr, nc, sg))
    return dict(trees=trees, init_score=init, F=F, train_loss=np.array(losses))


def engine_scale_bits(n_rows, w2, word_bits=126):
    """Fixed-point exponent S the CUDA engine uses for a round.

    Every |g| <= max(w) and every h <= max(w)/4, so with
    ``S = word_bits - 1 - ceil(log2(n_rows * max(w)))`` no partial sum of
    ``n_rows`` quantised values can reach 2^(word_bits-1).
    """
    wmax = float(np.max(w2))
    need = int(np.ceil(np.log2(max(1.0, n_rows * wmax)))) + 1
    return word_bits - 1 - need
