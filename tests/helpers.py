"""Shared helpers for the parity tests (loading fixtures, configs, comparing trees)."""
import ast
import os

import numpy as np

from conftest import GOLDEN


def golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def fit_inputs(name):
    """(X_train, y_train, X_test) of a golden fit, regenerated from its seeds."""
    from bsscl_gbm_b200 import datasets as D
    if name in ("cfg1", "cfg1_level", "mono"):
        Xtr, ytr, Xte, _ = D.config1()
        if name == "cfg1_level":
            return Xtr[:4000], ytr[:4000], Xte
        if name == "mono":
            return Xtr[:3000], ytr[:3000], Xte
        return Xtr, ytr, Xte
    if name == "cfg2_small":
        X, y = D.config2(n=40_000, n_pos=120)
        return X[:32_000], y[:32_000], X[32_000:]
    if name == "spw":
        X, y = D.config2(n=30_000, n_pos=150)
        return X[:24_000], y[:24_000], X[24_000:]
    if name == "cfg3_small":
        X, y = D.config3(n=25_000)
        return X[:20_000], y[:20_000], X[20_000:]
    if name == "reg":
        X, y = D.regression()
        return X[:6_400], y[:6_400], X[6_400:]
    if name == "mc":
        X, y = D.multiclass()
        return X[:6_400], y[:6_400], X[6_400:]
    if name == "cfg4_small":
        X, y = D.config4(n=30_000)
        return X[:24_000], y[:24_000], X[24_000:]
    raise KeyError(name)


def fit_params(d):
    return ast.literal_eval(str(d["params"]))


def oracle_fit_kwargs(d):
    params = fit_params(d)
    return dict(n_estimators=int(d["n_trees"]), learning_rate=float(d["learning_rate"]),
                max_leaves=int(d["max_leaves"]), max_depth=int(d["max_depth"]),
                min_samples_leaf=int(d["min_samples_leaf"]),
                min_child_weight=float(d["min_child_weight"]), reg_lambda=float(d["reg_lambda"]),
                gamma=float(d["gamma"]), subsample=float(d["subsample"]),
                colsample=float(d["colsample"]),
                class_weight=params.get("class_weight", "balanced_sqrt"),
                random_state=params["random_state"],
                grow_policy=params.get("grow_policy", "leaf"),
                scale_pos_weight=params.get("scale_pos_weight"), objective=params.get("objective", "auto"))


def golden_trees(d):
    out = []
    for t in range(int(d["n_trees"])):
        nc = int(d["nc"][t])
        out.append((d["tf"][t], d["tt"][t], d["tv"][t], d["tl"][t], d["tr"][t], nc, d["sg"][t]))
    return out


def golden_mc_trees(d):
    """Per class, the reference's trees of a multi-class fit fixture."""
    K, T = int(d["n_classes"]), int(d["n_trees"])
    return [[(d["tf"][k, t], d["tt"][k, t], d["tv"][k, t], d["tl"][k, t], d["tr"][k, t], int(d["nc"][k, t]),
              d["sg"][k, t]) for t in range(T)] for k in range(K)]


def reg_fit_kwargs(d):
    return dict(n_estimators=int(d["n_trees"]), learning_rate=float(d["learning_rate"]),
                max_leaves=int(d["max_leaves"]), max_depth=int(d["max_depth"]),
                min_samples_leaf=int(d["min_samples_leaf"]), min_child_weight=float(d["min_child_weight"]),
                reg_lambda=float(d["reg_lambda"]), gamma=float(d["gamma"]), subsample=float(d["subsample"]),
                colsample=float(d["colsample"]), random_state=0)


def mc_fit_kwargs(d):
    return dict(n_estimators=int(d["n_trees"]), learning_rate=float(d["learning_rate"]),
                max_leaves=int(d["max_leaves"]), max_depth=int(d["max_depth"]),
                min_samples_leaf=int(d["min_samples_leaf"]), min_child_weight=float(d["min_child_weight"]),
                reg_lambda=float(d["reg_lambda"]), gamma=float(d["gamma"]), subsample=float(d["subsample"]),
                colsample=float(d["colsample"]), class_weight="balanced_sqrt", random_state=0)


def same_topology(a, b):
    """tf/tt/tl/tr and node count identical."""
    na, nb = a[5], b[5]
    if na != nb:
        return False
    return all(np.array_equal(np.asarray(a[i])[:na], np.asarray(b[i])[:na]) for i in (0, 1, 3, 4))


def engine_scale_bits(wmax, chunk=16384):
    """Fixed-point exponent of the engine for weights up to ``wmax`` (libgbm_b200)."""
    return 62 - int(np.ceil(np.log2(chunk * max(1.0, wmax))))


def early_inputs():
    """(X_train, y_train, X_val, y_val, X_test) of tests/golden/fit_early.npz."""
    from bsscl_gbm_b200 import datasets as D
    X, y = D.config3(n=12_000)
    return X[:6000], y[:6000], X[6000:9000], y[6000:9000], X[9000:]


def val_loss(y, F):
    """The reference's binary log-loss (E:2321-2325)."""
    p = 1.0 / (1.0 + np.exp(-np.clip(F, -500, 500)))
    p = np.clip(p, 1e-15, 1 - 1e-15)
    return -np.mean(y * np.log(p) + (1 - y) * np.log(1 - p))
