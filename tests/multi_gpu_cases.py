"""The fits test_multi_gpu runs on 2 GPUs and on 1 (data, estimator arguments)."""


def _cfg3():
    from bsscl_gbm_b200 import datasets as D
    X, y = D.config3(n=25_000)
    return X[:20_000], y[:20_000], X[20_000:]


def _cfg4():
    from bsscl_gbm_b200 import datasets as D
    X, y = D.config4(n=30_000)
    return X[:24_000], y[:24_000], X[24_000:]


def _top():
    from bsscl_gbm_b200 import datasets as D
    X, y = D.top_bin(n=20_000)
    return X[:16_000], y[:16_000], X[16_000:]


CASES = {
    # the default constructor: 257 bin ids per feature, splits at threshold 255 (top cells summed over ranks)
    "top257": (_top, dict(n_estimators=8, random_state=0, verbose=False)),
    # the learned NaN direction
    "cfg4_nan": (_cfg4, dict(n_estimators=5, max_depth=6, n_bins=255, nan_direction="learn", random_state=5,
                             verbose=False)),
    # best-first, depth 6 (device replay of a fully speculated tree)
    "cfg3": (_cfg3, dict(n_estimators=12, max_depth=6, class_weight="balanced_sqrt", n_bins=255,
                         random_state=3, verbose=False)),
    # NaN in every feature, depth 8
    "cfg4_d8": (_cfg4, dict(n_estimators=6, max_depth=8, n_bins=255, random_state=1, verbose=False)),
    # depth-wise growth
    "cfg3_level": (_cfg3, dict(n_estimators=6, max_depth=5, grow_policy="level", n_bins=64,
                               class_weight="balanced", random_state=2, verbose=False)),
    # depth 12: capped speculation, replay on the host with on-demand expansion
    "cfg4_d12": (_cfg4, dict(n_estimators=3, max_depth=12, max_leaves=40, n_bins=255, random_state=4,
                             verbose=False)),
}
