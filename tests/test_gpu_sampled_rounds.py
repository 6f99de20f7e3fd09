"""The sampled multi-class and regression rounds (gbm_round_mc_sampled,
gbm_round_reg_sampled: the sampler's swap targets, with the shuffle, mask and
root row list built on the device) against the mask rounds (gbm_round_mc,
gbm_round_reg) fed the same sampler's host draw: the same trees, losses and
F, bit for bit, round after round, on a B200."""
import numpy as np
import pytest

import oracle as O
from helpers import fit_inputs, golden, mc_fit_kwargs, reg_fit_kwargs

pytestmark = pytest.mark.gpu

ROUNDS = 3


def _params(kw):
    from bsscl_gbm_b200 import GbmParams
    return GbmParams(kw["reg_lambda"], kw["gamma"], kw["min_child_weight"], kw["learning_rate"],
                     kw["min_samples_leaf"], kw["max_depth"], kw["max_leaves"], 0, None)


def _fields(t):
    nc = int(t[5])
    return [nc] + [np.asarray(t[i])[:nc].copy() for i in (0, 1, 2, 3, 4, 6)]


def _same(a, b):
    assert a[0] == b[0], f"{a[0]} vs {b[0]} nodes"
    for x, z in zip(a[1:], b[1:]):
        assert np.array_equal(x, z)


def _sampler(n, p, kw, seed):
    from bsscl_gbm_b200 import Sampler
    return Sampler(seed, n, p, int(n * kw["subsample"]), int(p * kw["colsample"]), True, True, look_ahead=2)


def test_mc_sampled_rounds_equal_mask_rounds():
    from bsscl_gbm_b200 import Engine
    d = golden("fit_mc")
    X, y, _ = fit_inputs("mc")
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    K = int(d["n_classes"])
    n, p = Xb.shape
    kw = mc_fit_kwargs(d)
    prm, cap = _params(kw), 2 * kw["max_leaves"] + 2
    w = O.class_weights_mc(y, K, "balanced_sqrt")
    runs = []
    for sampled in (True, False):
        eng = Engine(0)
        smp = _sampler(n, p, kw, 11)
        try:
            eng.upload_bins(Xb, d["counts"])
            eng.upload_labels_mc(y.astype(np.uint8), K, w)
            got = []
            for _ in range(ROUNDS):
                if sampled:
                    trees, loss = eng.round_mc_sampled(smp, 0, prm, cap)
                else:
                    _, mask, feat = smp.next(want_sample=False, want_mask=True)
                    trees, loss, _ = eng.round_mc(mask, feat, prm, cap)
                got.append(([_fields(t) for t in trees], loss))
            runs.append((got, eng.get_F_mc()))
        finally:
            smp.close()
            eng.close()
    (a, Fa), (b, Fb) = runs
    for r in range(ROUNDS):
        assert a[r][1] == b[r][1], f"round {r} loss"
        for k in range(K):
            _same(a[r][0][k], b[r][0][k])
    assert np.array_equal(Fa, Fb)


@pytest.mark.parametrize("loss", ["mse", "mae"])
def test_reg_sampled_rounds_equal_mask_rounds(loss):
    from bsscl_gbm_b200 import Engine
    d = golden(f"fit_reg_{loss}")
    X, y, _ = fit_inputs("reg")
    Xb = O.bin_matrix(X, d["edges"], d["counts"], d["nan_bin_id"], False)
    n, p = Xb.shape
    kw = reg_fit_kwargs(d)
    prm, cap = _params(kw), 2 * kw["max_leaves"] + 2
    runs = []
    for sampled in (True, False):
        eng = Engine(0)
        smp = _sampler(n, p, kw, 13)
        try:
            eng.upload_bins(Xb, d["counts"])
            eng.upload_targets(y, float(np.mean(y)), loss)
            got = []
            for _ in range(ROUNDS):
                if sampled:
                    tree, tloss = eng.round_reg_sampled(smp, 0, prm, cap)
                else:
                    _, mask, feat = smp.next(want_sample=False, want_mask=True)
                    tree, tloss, _ = eng.round_reg(mask, feat, prm, cap)
                got.append((_fields(tree), tloss))
            runs.append((got, eng.get_F()))
        finally:
            smp.close()
            eng.close()
    (a, Fa), (b, Fb) = runs
    for r in range(ROUNDS):
        assert a[r][1] == b[r][1], f"round {r} loss"
        _same(a[r][0], b[r][0])
    assert np.array_equal(Fa, Fb)
