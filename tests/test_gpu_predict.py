"""k_predict (the ensemble walk, predict_all_trees_jit E:863-884 + the sigmoid
of predict_proba E:3318-3336) against the CPU oracle, over every shape the
kernel chooses between:

* the row tile: two rows per thread (p <= 100), one row per thread with
  fewer rows per CTA (p = 200, 5000), rows read from global memory when a
  32-row tile no longer fits shared memory (p = 9000), and the byte-wise
  tile load when p is not a multiple of 4;
* the node format: 32-bit breadth-first words (p <= 4096 and trees of at
  most 4096 nodes) or 8-byte nodes in the reference's own numbering;
* the chunks: trees larger than the 2048-node shared buffer, walked from
  global memory, between small ones; many one-leaf trees in one chunk;
* tree numbering: the reference's non-adjacent children (depth-first
  preorder here), renumbered breadth-first on upload.

F must agree with the oracle to 1e-12 (the sum runs in the same tree order;
the leaf product lr * value is rounded the same way).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _preorder_tree(rng, n_internal, p, max_thr=255):
    """A random binary tree with ``n_internal`` splits, numbered in
    depth-first preorder: the left child is the next id and the right child
    comes after the whole left subtree (children after their parent, never
    adjacent to each other unless the left child is a leaf)."""
    # random shape: each split has k internal nodes below it, split at random
    def build(k):
        if k == 0:
            return None
        kl = int(rng.integers(0, k))
        return (build(kl), build(k - 1 - kl))

    shape = build(n_internal)
    feat, thr, left, right, val = [], [], [], [], []

    def emit(s):
        i = len(feat)
        feat.append(-1), thr.append(0), left.append(-1), right.append(-1), val.append(rng.normal(0, 0.1))
        if s is None:
            return i
        feat[i] = int(rng.integers(0, p))
        thr[i] = int(rng.integers(0, max_thr + 1))
        left[i] = emit(s[0])
        right[i] = emit(s[1])
        return i

    emit(shape)
    return feat, thr, val, left, right


def _ensemble_from_trees(trees):
    feats, thrs, vals, lefts, rights, offs = [], [], [], [], [], [0]
    for f, t, v, l, r in trees:
        feats += f
        thrs += t
        vals += v
        lefts += l
        rights += r
        offs.append(offs[-1] + len(f))
    return {"features": np.array(feats, np.int16), "thresholds": np.array(thrs, np.int64),
            "values": np.array(vals, np.float64), "left": np.array(lefts, np.int32),
            "right": np.array(rights, np.int32), "offsets": np.array(offs, np.int32)}


def _check(engine, Xb, ens, n_trees, lr=0.08, base=-0.7):
    F, P = engine.predict(Xb, ens, n_trees, lr, base)
    Fo = O.predict_packed(Xb, ens, n_trees, lr) + base
    assert np.abs(F - Fo).max() <= 1e-12
    assert np.abs(P - 1.0 / (1.0 + np.exp(-np.clip(Fo, -500, 500)))).max() <= 1e-12


@pytest.mark.parametrize("p", [37, 100, 200, 5000])
def test_predict_row_tile_shapes(engine, p):
    from bsscl_gbm_b200 import datasets as D
    rng = np.random.default_rng(p)
    n = 3000 if p < 1000 else 700
    Xb = rng.integers(0, 256, size=(n, p)).astype(np.uint8)
    ens = D.config5_ensemble(n_trees=30, depth=8, p=p, seed=p)
    _check(engine, Xb, ens, 30)


def test_predict_rows_too_wide_for_shared_memory(engine):
    """p = 9000: a 32-row tile would need 288 KB, so rows are read from
    global memory; features > 4096 also select the 8-byte node format."""
    rng = np.random.default_rng(1)
    n, p = 500, 9000
    Xb = rng.integers(0, 256, size=(n, p)).astype(np.uint8)
    trees = [_preorder_tree(rng, 40, p) for _ in range(12)]
    _check(engine, Xb, _ensemble_from_trees(trees), 12)


def test_predict_preorder_trees_and_oversize_chunks(engine):
    """Depth-first numbered trees (non-adjacent children), including two of
    3001 and 4501 nodes (larger than the 2048-node chunk buffer, so walked
    from global memory; the second is also past the 32-bit format's 4096-node
    limit, so the whole model keeps the 8-byte format), between small trees
    and a run of one-leaf trees."""
    rng = np.random.default_rng(2)
    n, p = 4000, 48
    Xb = rng.integers(0, 256, size=(n, p)).astype(np.uint8)
    small = [_preorder_tree(rng, int(rng.integers(1, 60)), p) for _ in range(20)]
    leaf = [([-1], [0], [float(rng.normal())], [-1], [-1]) for _ in range(700)]
    big = [_preorder_tree(rng, 1500, p)]
    trees = small[:10] + big + leaf + small[10:]
    _check(engine, Xb, _ensemble_from_trees(trees), len(trees))
    huge = [_preorder_tree(rng, 2250, p)]
    trees2 = small[:5] + huge + small[5:]
    _check(engine, Xb, _ensemble_from_trees(trees2), len(trees2))


def test_predict_thresholds_above_the_bin_range(engine):
    """A threshold above 255 sends every uint8 bin left, as the reference's
    compare does (the engine stores it as 255)."""
    rng = np.random.default_rng(3)
    n, p = 2000, 16
    Xb = rng.integers(0, 256, size=(n, p)).astype(np.uint8)
    trees = [_preorder_tree(rng, 30, p, max_thr=300) for _ in range(8)]
    _check(engine, Xb, _ensemble_from_trees(trees), 8)
