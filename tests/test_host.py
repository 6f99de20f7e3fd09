"""Host-side logic that needs no GPU: binning, sampler, the C-ABI library's
exports, estimator argument handling, and that nothing falls back to a CPU
path when no device is present."""
import glob
import hashlib
import os
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from helpers import fit_inputs, golden


@pytest.mark.parametrize("case", sorted(os.path.basename(f)[:-4]
                                        for f in glob.glob(os.path.join(GOLDEN, "bin_*.npz"))))
def test_host_edges_and_bins_match_reference(case):
    from bsscl_gbm_b200 import binning
    d = golden(case)
    e, c, nb = binning.build_bin_edges(d["X"], int(d["n_bins"]))
    assert np.array_equal(e, d["edges"])
    assert np.array_equal(c, d["counts"])
    assert np.array_equal(nb, d["nan_bin_id"])
    Xb = binning.bin_features(d["X"], d["edges"], d["counts"], d["nan_bin_id"])
    assert np.array_equal(Xb, d["X_bin"])


@pytest.mark.parametrize("name", ["cfg1", "cfg2_small", "cfg3_small", "cfg4_small"])
def test_host_binning_of_fit_inputs(name):
    from bsscl_gbm_b200 import binning
    d = golden("fit_" + name)
    X, _, _ = fit_inputs(name)
    e, c, nb = binning.build_bin_edges(X, int(d["n_bins"]))
    assert np.array_equal(e, d["edges"]) and np.array_equal(c, d["counts"])
    Xb = binning.bin_features(X, e, c, nb)
    assert hashlib.sha256(Xb.astype(np.uint16).tobytes()).hexdigest() == str(d["X_bin_sha"])


def test_device_bins_clamp_is_lossless():
    """ids >= bin_count (the float32 max-edge quirk) clamp to bin_count-1."""
    import oracle as O
    from bsscl_gbm_b200 import binning
    rng = np.random.default_rng(3)
    X = rng.integers(0, 7, size=(2000, 3)).astype(np.float32)    # few levels, float32
    X[rng.random((2000, 3)) < 0.2] = np.nan                        # NaN bin on every column
    e, counts, nb = binning.build_bin_edges(X, 255)
    raw = binning.bin_features(X, e, counts, nb)
    assert np.array_equal(raw, O.bin_matrix(X, e, counts, nb, False))
    assert (raw >= counts[None, :]).any()           # the quirk is present
    dev = binning.device_bins(raw, counts)
    assert dev.dtype == np.uint8
    assert np.array_equal(dev, np.minimum(raw, counts - 1))
    # every threshold the reference can pick (<= nb-2) routes raw and clamped ids alike
    for j in range(raw.shape[1]):
        for thr in range(max(0, counts[j] - 1)):
            assert np.array_equal(raw[:, j] <= thr, dev[:, j] <= thr)


def test_sampler_matches_numpy_randomstate(built_lib):
    from bsscl_gbm_b200 import Sampler
    d = np.load(os.path.join(GOLDEN, "sampler.npz"))
    for seed, n, p, frac, fc, rounds in [(0, 1000, 30, 0.8, 0.8, 5), (7, 70000, 100, 0.75, 0.7, 3),
                                         (4294967295, 17, 3, 0.5, 0.5, 4)]:
        ns, nf = max(1, int(n * frac)), max(1, int(p * fc))
        for ahead in (0, 2):
            s = Sampler(seed, n, p, ns, nf, True, True, look_ahead=ahead)
            for r in range(rounds):
                smp, mask, feat = s.next(want_sample=True, want_mask=True)
                assert np.array_equal(smp, d[f"s{seed}_n{n}_r{r}_sample"])
                assert np.array_equal(feat, d[f"s{seed}_n{n}_r{r}_feat"])
                assert mask.sum() == ns and mask[smp].all()
            s.close()


def test_sampler_matches_numpy_at_full_size(built_lib):
    """1M rows (every mask width of the bounded draw, the vectorised blocks
    and their word-by-word fallback) against NumPy's RandomState itself."""
    from bsscl_gbm_b200 import Sampler
    n, p = 1_000_000, 100
    rs = np.random.RandomState(11)
    rows, feats = np.arange(n), np.arange(p, dtype=np.int32)
    s = Sampler(11, n, p, 750_000, 70, True, True, look_ahead=2)
    for _ in range(2):
        rs.shuffle(rows)
        rs.shuffle(feats)
        smp, _, feat = s.next(want_sample=True, want_mask=False)
        assert np.array_equal(smp, rows[:750_000])
        assert np.array_equal(feat, np.sort(feats[:70]))
    s.close()


def test_sampler_avx512_and_avx2_paths_agree(built_lib):
    """The sampler's AVX-512 twist/draw (used where the CPU has it) and its
    AVX2 versions give the same stream: compare this process with a child
    forced onto the AVX2 versions."""
    import subprocess
    import sys
    from bsscl_gbm_b200 import Sampler
    code = ("import sys; sys.path.insert(0, %r); import numpy as np; from bsscl_gbm_b200 import Sampler; "
            "s = Sampler(5, 300001, 40, 200000, 30, True, True, look_ahead=2); "
            "out = [s.next(want_sample=True, want_mask=False) for _ in range(3)]; "
            "np.savez(sys.argv[1], *[a for o in out for a in (o[0], o[2])])" % os.path.join(ROOT, "bsscl-gbm_b200"))
    import tempfile
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "avx2.npz")
        env = dict(os.environ, GBM_SAMPLER_ISA="avx2")
        subprocess.run([sys.executable, "-c", code, path], env=env, check=True, timeout=120)
        ref = np.load(path)
        s = Sampler(5, 300001, 40, 200000, 30, True, True, look_ahead=2)
        got = [a for _ in range(3) for a in (lambda o: (o[0], o[2]))(s.next(want_sample=True, want_mask=False))]
        s.close()
        for k, a in enumerate(got):
            assert np.array_equal(a, ref[f"arr_{k}"])


def _fisher_yates(n, j):
    a = np.arange(n)
    for i in range(n - 1, 0, -1):
        a[i], a[j[i]] = a[j[i]], a[i]
    return a


def _shuffle_from_targets(n, j):
    """The engine's parallel construction of a round's shuffle (gbm_kernels.cuh,
    k_shuf_link / k_shuf_min / k_shuf_compose), restated with NumPy."""
    steps = np.arange(1, n)
    order = np.lexsort((steps, j[1:]))                 # steps grouped by target, ascending
    tgt, st = j[1:][order], steps[order]
    m = np.full(n, -1)                                 # m(q): smallest step > q targeting q
    mp = np.full(n, -1)                                # mp(i): next larger step with i's target
    same = tgt[1:] == tgt[:-1]
    mp[st[:-1][same]] = st[1:][same]
    above = st > tgt
    first = np.ones(len(st), bool)
    first[1:] = ~(same & above[:-1] & above[1:])
    sel = above & first
    for q, i in zip(tgt[sel], st[sel]):
        if m[q] < 0:
            m[q] = i
    def root(i):
        while m[i] >= 0:
            i = m[i]
        return i
    S = np.empty(n, np.int64)
    S[0] = root(m[0]) if m[0] >= 0 else 0
    for i in range(1, n):
        S[i] = root(mp[i]) if mp[i] >= 0 else j[i]
    return S


@pytest.mark.parametrize("n", [1, 2, 3, 17, 1000, 20000])
def test_parallel_shuffle_construction_equals_fisher_yates(n):
    rng = np.random.default_rng(n)
    for _ in range(3):
        j = np.zeros(n, np.int64)
        for i in range(1, n):
            j[i] = rng.integers(0, i + 1)
        assert np.array_equal(_shuffle_from_targets(n, j), _fisher_yates(n, j))


def test_sampler_matches_fit_stream(built_lib):
    """The per-round sample hashes the reference recorded during its fit."""
    from bsscl_gbm_b200 import Sampler
    d = golden("fit_cfg1")
    n = 10_000
    s = Sampler(0, n, 30, int(n * float(d["subsample"])), int(30 * float(d["colsample"])), True, True)
    for t in range(int(d["n_trees"])):
        smp, _, _ = s.next(want_sample=True, want_mask=False)
        assert hashlib.sha256(smp.tobytes()).hexdigest() == str(d["sample_sha"][t])
    s.close()


def test_library_exports_every_declared_symbol(built_lib):
    import ctypes
    from bsscl_gbm_b200 import _lib
    hdr = open(os.path.join(ROOT, "include", "gbm_b200.h")).read()
    declared = set(re.findall(r"\b(gbm_[A-Za-z0-9_]+)\s*\(", hdr))
    assert declared, "no declarations parsed"
    L = ctypes.CDLL(built_lib)
    missing = [s for s in sorted(declared) if not hasattr(L, s)]
    assert not missing, missing
    assert declared == set(_lib.EXPORTS)


def test_no_device_raises_instead_of_falling_back(built_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from bsscl_gbm_b200 import Engine, HybridHistGBMNumbaV1_0_1
    with pytest.raises(RuntimeError):
        Engine(0)
    X = np.random.default_rng(0).standard_normal((200, 4))
    y = (X[:, 0] > 0).astype(int)
    with pytest.raises(RuntimeError):
        HybridHistGBMNumbaV1_0_1(n_estimators=2, verbose=False, random_state=0).fit(X, y)


def test_estimator_argument_errors():
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    X = np.random.default_rng(0).standard_normal((100, 5))
    y = np.random.default_rng(1).integers(0, 2, 100)
    with pytest.raises(ValueError):
        M(max_depth=-5, verbose=False).fit(X, y)
    with pytest.raises(ValueError):
        M(learning_rate=-0.1, verbose=False).fit(X, y)
    with pytest.raises(ValueError):
        M(n_estimators=0, verbose=False).fit(X, y)
    with pytest.raises(ValueError):
        M(verbose=False).fit(X, y[:99])
    with pytest.raises(ValueError):
        M(verbose=False).predict(X)
    with pytest.raises(ValueError):
        M(device="cpu")
    with pytest.raises(NotImplementedError):
        M(objective="regression", loss="huber", verbose=False).fit(X, y)
    with pytest.raises(NotImplementedError):
        M(sampling_method="goss", verbose=False).fit(X, y)
    with pytest.raises(NotImplementedError):
        M(verbose=False).fit(X, np.arange(100) % 65)   # more classes than the engine holds
    # the reference's own fuzz cases that fail before training (T:test_fuzz.py:5-31)
    with pytest.raises((ValueError, TypeError)):
        M(n_estimators=1, max_depth=2, verbose=False).fit(np.array([["a", "b"], ["c", "d"]]), np.array([0, 1]))
    with pytest.raises((ValueError, IndexError)):
        M(n_estimators=1, max_depth=2, verbose=False).fit(np.array([[]]), np.array([]))
    with pytest.raises(ValueError):
        M(n_estimators=1, max_depth=2, verbose=False).fit(np.zeros((0, 3)), np.zeros(0))


def test_adaptive_hyperparameters_follow_reference():
    """'auto' resolution, checked against the values the reference recorded."""
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    for name in ("cfg1", "cfg2_small", "cfg3_small", "cfg4_small"):
        d = golden("fit_" + name)
        X, y, _ = fit_inputs(name)
        from helpers import fit_params
        m = M(verbose=False, **fit_params(d))
        m._compute_adaptive_hyperparameters(X, y)
        assert m.learning_rate == float(d["learning_rate"])
        assert m.max_leaves == int(d["max_leaves"])
        assert m.max_depth == int(d["max_depth"])
        assert m.min_child_weight == float(d["min_child_weight"])
        assert m.subsample == float(d["subsample"])
        assert m.colsample_bytree == float(d["colsample"])
        assert m.reg_lambda == float(d["reg_lambda"])
        assert m.binning_strategy == str(d["binning_strategy"])


def test_get_set_params_roundtrip():
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    m = M(n_estimators=7, max_depth=3, verbose=False)
    p = m.get_params()
    assert p["n_estimators"] == 7 and p["max_depth"] == 3 and p["device"] == "b200"
    m.set_params(learning_rate=0.3)
    assert m.learning_rate == 0.3
    with pytest.raises(ValueError):
        m.set_params(bogus=1)


def test_c_abi_rejects_bad_arguments_without_a_device(built_lib):
    """Argument checks of the binning, multi-class, regression and self-test
    entry points run before any CUDA call: on a host without a GPU they
    answer GBM_ERR_ARG (1) for null contexts and out-of-range values."""
    import ctypes as C
    from bsscl_gbm_b200 import _lib
    L = _lib.lib()
    GBM_ERR_ARG = 1
    assert L.gbm_bin_edges(None, None, 0, 0, 0, 255, None, None, 0, None, None, None) == GBM_ERR_ARG
    assert L.gbm_upload_binned_rows(None, 0, 1, None, 0, None, None) == GBM_ERR_ARG
    assert L.gbm_bin_features(None, None, 1, 1, 0, None, 0, None, None, None) == GBM_ERR_ARG
    assert L.gbm_predict_upload_raw(None, None, 1, 1, 0, None, 0, None, None) == GBM_ERR_ARG
    assert L.gbm_upload_labels_mc(None, None, 3, None, 0) == GBM_ERR_ARG
    assert L.gbm_round_mc(None, None, None, 1, None, None, None) == GBM_ERR_ARG
    assert L.gbm_upload_targets(None, None, 0.0, 0, 0) == GBM_ERR_ARG
    assert L.gbm_round_reg(None, None, None, 1, None, None, None) == GBM_ERR_ARG
    assert L.gbm_get_grad_mc(None, 0, None, None) == GBM_ERR_ARG
    assert L.gbm_test_peer_wait(0, 0) == GBM_ERR_ARG          # the limit must be 1..10000 ms
    assert L.gbm_test_peer_wait(0, 20000) == GBM_ERR_ARG


def test_malformed_models_are_rejected_on_the_host(built_lib):
    """gbm_check_model -- the checks gbm_predict_set_model runs before any
    upload or launch -- accepts a well-formed ensemble and rejects every
    model whose walk could loop or leave its tree: a child at or before its
    parent (a cycle), a child past the tree's end, offsets that start below 0,
    an empty tree, a feature >= p and a negative threshold."""
    from bsscl_gbm_b200 import datasets as D
    from bsscl_gbm_b200._lib import check_model
    good = D.config5_ensemble(n_trees=4, depth=3, p=10, seed=1)
    check_model(good, 4, 10)

    def bad(mutate, msg):
        m = {k: v.copy() for k, v in good.items()}
        mutate(m)
        with pytest.raises(ValueError, match=msg):
            check_model(m, 4, 10)

    bad(lambda m: m["left"].__setitem__(15 + 2, 2), "must lie after")     # tree 1, node 2 -> itself
    bad(lambda m: m["right"].__setitem__(0, 0), "must lie after")         # root -> root: a cycle
    bad(lambda m: m["left"].__setitem__(3, 40), "must lie after")         # past the tree's end
    bad(lambda m: m["offsets"].__setitem__(0, -5), "start at -5")
    bad(lambda m: m["offsets"].__setitem__(2, m["offsets"][1]), "empty")
    bad(lambda m: m["features"].__setitem__(1, 10), "feature 10 >= 10")
    bad(lambda m: m["thresholds"].__setitem__(2, -1), "negative threshold")


def _rot_bytes(words, r):
    """k_hist3's rot_bytes on four 32-bit words: byte k of the result is byte
    (k + r) mod 16 of the input (restated with NumPy for the check below)."""
    a, b, c, d = words
    if r & 8:
        a, b, c, d = c, d, a, b
    if r & 4:
        a, b, c, d = b, c, d, a
    sh = (r & 3) * 8

    def fsr(lo, hi):
        return int(((hi << 32) | lo) >> sh) & 0xFFFFFFFF
    return fsr(a, b), fsr(b, c), fsr(c, d), fsr(d, a)


def test_hist3_layout_is_conflict_free_and_complete():
    """The shared-memory layout of k_hist3 (csrc/gbm_kernels.cuh): in step k
    lane l = 16 h + f adds feature (f + k) mod 16 into word
    ((digit * 257 + bin) * 2 + h) * 16 + (f + k) mod 16, where bin is the
    row's bin, or 256 (the trash row) when the round did not select that
    feature.  For every step and any bins and selection, the 32 lanes use 32
    different banks; over 16 steps every lane adds each of the 16 features
    of its row exactly once; every word lies inside the 6 x 257 x 32-word
    accumulator; and the byte each lane reads from its rotated record is
    that feature's bin."""
    rng = np.random.default_rng(0)
    kBlk, kDigV3 = 16, 257 * 2 * 16
    for _ in range(200):
        bins = rng.integers(0, 256, size=(32, kBlk))          # the 16 bins of each lane's row
        sel = rng.random(kBlk) < 0.7                          # the round's selected features of the block
        digit = int(rng.integers(0, 6))
        seen = np.zeros((32, kBlk), dtype=int)
        for k in range(kBlk):
            banks = set()
            for lane in range(32):
                h, f = lane >> 4, lane & 15
                feat = (f + k) & (kBlk - 1)
                seen[lane, feat] += 1
                b = int(bins[lane, feat]) if sel[feat] else 256
                word = digit * kDigV3 + (b * 2 + h) * kBlk + feat
                assert 0 <= word < 6 * kDigV3
                banks.add(word % 32)
            assert len(banks) == 32
        assert np.all(seen == 1)
    for _ in range(300):
        by = rng.integers(0, 256, size=16)
        words = tuple(int(sum(int(by[4 * i + j]) << (8 * j) for j in range(4))) for i in range(4))
        r = int(rng.integers(0, 16))
        out = _rot_bytes(words, r)
        for k in range(16):
            assert (out[k >> 2] >> ((k & 3) * 8)) & 0xFF == by[(k + r) % 16]


def _partition_restated(rows, left, begin, end, tile=4096, threads=512):
    """k_partition's index arithmetic for one task, restated: position o of
    tile k is word (o >> 5) = warp + j * (threads / 32) with lane o & 31; a
    left goes to begin + lcar + lrank, a right to end - 1 - rcar - (o - lrank)."""
    out = np.full(len(rows), -1, dtype=np.int64)
    lcar = 0
    ntile = max(1, -(-(end - begin) // tile))
    for k in range(ntile):
        r0 = begin + k * tile
        m = min(tile, end - r0)
        l = np.zeros(tile, bool)
        l[:m] = left[r0:r0 + m]
        words = l.reshape(tile // 32, 32)
        pre = np.concatenate([[0], np.cumsum(words.sum(axis=1))[:-1]])
        rcar = (r0 - begin) - lcar
        for o in range(m):
            lrank = pre[o >> 5] + int(words[o >> 5, :(o & 31)].sum())
            dst = begin + lcar + lrank if l[o] else end - 1 - rcar - (o - lrank)
            assert begin <= dst < end and out[dst] == -1
            out[dst] = rows[r0 + o]
        lcar += int(l[:m].sum())
    return out[begin:end], lcar


def _best_first_splits(gain, valid, kids, max_leaves, gamma):
    """The reference's best-first loop (E:642-801) over a fully grown tree:
    split the candidate of largest gain (> gamma) while fewer than
    max_leaves - 1 splits are made; a split that cannot be made (min_samples_leaf)
    turns the candidate into a leaf.  Returns the nodes split."""
    cand, done = [0], []
    while len(done) < max_leaves - 1:
        live = [c for c in cand if gain[c] > gamma]
        if not live:
            break
        best = max(gain[c] for c in live)
        v = min(c for c in live if gain[c] == best)
        cand.remove(v)
        if not valid[v] or kids[v] is None:
            continue
        done.append(v)
        cand.extend(kids[v])
    return set(done)


def _prunable(v, gain, valid, parent, depth, known, max_leaves, gamma):
    """k_level_close / k_partition's rule for node v, counting only the nodes
    whose splits are known (`known`): v is skipped when its depth plus the
    other known nodes whose whole path is of makeable splits with gains above
    v's reach max_leaves - 1."""
    def mg(w):
        m = np.inf
        while w >= 0:
            if not (known[w] and valid[w] and gain[w] > gamma):
                return -np.inf
            m = min(m, gain[w])
            w = parent[w]
        return m
    anc = set()
    a = parent[v]
    while a >= 0:
        anc.add(a)
        a = parent[a]
    cnt = sum(1 for w in range(len(gain)) if w != v and w not in anc and known[w] and mg(w) > gain[v])
    return depth[v] + cnt >= max_leaves - 1


def _prune_case(seed):
    """One random complete tree and the pruning rule checked on it; returns
    how many (node, stage) pairs the rule skipped."""
    rng = np.random.default_rng(seed)
    D = int(rng.integers(5, 9))
    N = 2 ** (D + 1) - 1
    parent = np.array([-1] + [(i - 1) // 2 for i in range(1, N)])
    depth = np.array([int(np.floor(np.log2(i + 1))) for i in range(N)])
    gain = np.round(rng.exponential(1.0, N) * np.exp(-0.3 * depth), 1)   # rounding makes ties
    valid = rng.random(N) > 0.1
    kids = [(2 * i + 1, 2 * i + 2) if 2 * i + 2 < N else None for i in range(N)]
    max_leaves = int(rng.integers(3, 40))
    gamma = float(rng.choice([0.0, 0.2]))
    split = _best_first_splits(gain, valid, kids, max_leaves, gamma)
    skipped = 0
    for v in range(1, N):
        at_close = depth < depth[v]     # partitioned when v's parent level closes
        after_part = depth <= depth[v]  # v's own level partitioned too
        for known in (at_close, after_part):
            if _prunable(v, gain, valid, parent, depth, known, max_leaves, gamma):
                assert v not in split, (seed, v)
                skipped += 1
        # after the partition a parent under (or with) a split that cannot be made drops out too
        w, reach = v, True
        while w >= 0:
            reach &= bool(valid[w] and gain[w] > gamma)
            w = parent[w]
        if not reach:
            assert v not in split, (seed, v)
    return skipped


@pytest.mark.parametrize("seed", range(40))
def test_best_first_pruning_never_skips_a_node_the_loop_splits(seed):
    """On random complete trees (depth 5-8, ties, unmakeable splits, gains
    that rise below their parents), every node the pruning rule skips -- with
    the nodes above its level known (the level close) or its own level too
    (after the partition) -- is one the best-first loop never splits."""
    _prune_case(seed)


def test_best_first_pruning_is_not_vacuous():
    assert sum(_prune_case(seed) for seed in range(40)) > 100


@pytest.mark.parametrize("size", [1, 31, 4096, 4097, 20_000])
def test_partition_index_arithmetic_is_a_monotonic_permutation(size):
    """Every row lands once inside the task's range, the lefts first in list
    order and the rights after them in reverse order, so an ascending list
    gives an ascending left child and a descending right child (and a
    monotonic list gives monotonic children at every depth)."""
    rng = np.random.default_rng(size)
    begin = 7
    rows = np.concatenate([np.full(begin, -5), np.sort(rng.choice(10 * size + 10, size, replace=False)),
                           np.full(3, -9)])
    left = rng.random(len(rows)) < 0.4
    out, nl = _partition_restated(rows, left, begin, begin + size)
    seg, lseg = rows[begin:begin + size], left[begin:begin + size]
    assert nl == int(lseg.sum())
    assert np.array_equal(out[:nl], seg[lseg])
    assert np.array_equal(out[nl:], seg[~lseg][::-1])
    # the right child, partitioned again, stays monotonic (descending in, so left part descending)
    if size - nl > 1:
        r = out[nl:]
        l2 = rng.random(len(r)) < 0.5
        out2, nl2 = _partition_restated(r, l2, 0, len(r))
        assert np.all(np.diff(out2[:nl2]) < 0) and np.all(np.diff(out2[nl2:]) > 0)


@pytest.mark.parametrize("name", ["cfg1", "cfg1_level", "cfg2_small", "cfg3_small", "cfg4_small"])
def test_packing_and_importances_match_reference(name):
    """The estimator's packing (_pack_tree_list, E:2192-2216) and gain
    importances (E:2343-2363), given the reference's own trees of a recorded
    fit, equal the reference's packed arrays and feature_importances_."""
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    from helpers import golden_trees
    d = golden("fit_" + name)
    X, _, _ = fit_inputs(name)
    m = M(verbose=False)
    m.trees = golden_trees(d)
    m.mc_trees = None
    m._is_multiclass = False
    m.n_features_in_ = X.shape[1]
    m._pack_trees()
    m._compute_feature_importances()
    for mine, ref in (("_packed_features", "packed_features"), ("_packed_thresholds", "packed_thresholds"),
                      ("_packed_values", "packed_values"), ("_packed_left", "packed_left"),
                      ("_packed_right", "packed_right"), ("_tree_offsets", "tree_offsets")):
        assert np.array_equal(getattr(m, mine), d[ref]), mine
        assert getattr(m, mine).dtype == d[ref].dtype, mine
    assert np.array_equal(m.feature_importances_, d["feature_importances"])


def test_pickle_round_trip_of_a_fitted_model():
    """A model holding a recorded fit survives pickle (T:test_serialization.py:9-35):
    trees, packed arrays, edges and hyper-parameters come back equal, and the
    device handle is not pickled."""
    import pickle
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1 as M
    from helpers import golden_trees, fit_params
    d = golden("fit_cfg3_small")
    X, _, _ = fit_inputs("cfg3_small")
    m = M(verbose=False, **fit_params(d))
    m.trees = golden_trees(d)
    m.mc_trees = None
    m._is_multiclass = False
    m.n_features_in_ = X.shape[1]
    m.bin_edges, m.feature_bin_counts, m._nan_bin_id = d["edges"], d["counts"], d["nan_bin_id"]
    m.base_score_ = float(d["base_score"])
    m._pack_trees()
    m._compute_feature_importances()
    m._engine = object()            # stands in for a live device context
    b = pickle.loads(pickle.dumps(m))
    assert b._engine is None
    assert b.get_params() == m.get_params()
    for ta, tb in zip(m.trees, b.trees):
        for x, y in zip(ta, tb):
            assert np.array_equal(np.asarray(x), np.asarray(y))
    for k in ("_packed_features", "_packed_thresholds", "_packed_values", "_packed_left", "_packed_right",
              "_tree_offsets", "bin_edges", "feature_bin_counts", "_nan_bin_id", "feature_importances_"):
        assert np.array_equal(getattr(m, k), getattr(b, k)), k
    assert b.base_score_ == m.base_score_


# --- the ranked (parallel) form of the device's best-first replay -----------

def _order_key(g):
    """k_replay_leaf's order_key: a double as an unsigned key of the same order."""
    import struct
    u = struct.unpack("<Q", struct.pack("<d", float(g)))[0]
    return (~u) & (2 ** 64 - 1) if u >> 63 else u | (1 << 63)


def _replay_loop(T, max_leaves, gamma, msl, max_depth):
    """k_replay_leaf's warp loop restated (candidate slots, lowest slot first
    on equal keys, the two lowest free slots, E:642-823).  T: list of dicts
    (feat, gain, n, local, kid0, kid1, expanded, depth, parent).  Returns
    (status, nc, {tree id: ('split', node, lid, rid) | ('leaf', node)}, alg)."""
    ck = lambda x: _order_key(x["gain"]) if x["feat"] >= 0 and x["gain"] > gamma else 0
    MAXC = max_leaves + 2
    key, act = [0] * MAXC, [False] * MAXC
    c_node, c_nid = [0] * MAXC, [0] * MAXC
    key[0], act[0] = ck(T[0]), True
    nc, ns, status, out, alg = 1, 0, 0, {}, T[0]["local"]
    while ns < max_leaves - 1:
        best = max(key)
        if best == 0:
            break
        ci = key.index(best)
        cur, pn = c_node[ci], T[c_nid[ci]]
        if not pn["expanded"]:
            status = 1
            break
        gnl, gnr = T[pn["kid0"]]["n"], T[pn["kid1"]]["n"]
        if gnl < msl or gnr < msl:
            out[cur] = ("leaf", c_nid[ci])
            key[ci], act[ci] = 0, False
            continue
        ss, sl = [s for s in range(MAXC) if s != ci and not act[s]][:2]
        lid, rid = nc, nc + 1
        nc += 2
        ns += 1
        small = gnl <= gnr
        kid_s, kid_l = (pn["kid0"], pn["kid1"]) if small else (pn["kid1"], pn["kid0"])
        if pn["depth"] + 1 < max_depth:
            alg += T[kid_s]["local"]
        out[cur] = ("split", c_nid[ci], lid, rid)
        c_node[ss], c_nid[ss] = (lid if small else rid), kid_s
        c_node[sl], c_nid[sl] = (rid if small else lid), kid_l
        key[ci], act[ci] = 0, False
        key[ss], act[ss] = ck(T[kid_s]), True
        key[sl], act[sl] = ck(T[kid_l]), True
    if not status:
        for s in range(MAXC):
            if act[s]:
                out[c_node[s]] = ("leaf", c_nid[s])
    return status, nc, out, alg


def _replay_ranked(T, max_leaves, gamma, msl, max_depth, max_c=256, max_d=15):
    """k_replay_leaf's ranked path restated: the candidates C (key > 0, every
    ancestor a makeable split), u before v when u is v's ancestor or, below
    their lowest common ancestor, u's path has the larger smallest key; a
    split's rank is the number of makeable candidates before it.  None where
    the kernel hands over to the loop (equal keys among C, an unexpanded
    candidate the loop would reach, too many candidates or too deep)."""
    ck = lambda x: _order_key(x["gain"]) if x["feat"] >= 0 and x["gain"] > gamma else 0
    mk = lambda x: (ck(x) != 0 and x["expanded"] and T[x["kid0"]]["n"] >= msl and T[x["kid1"]]["n"] >= msl)
    K = max_leaves - 1
    C = []
    for i, x in enumerate(T):
        if ck(x) == 0:
            continue
        a = x["parent"]
        while a >= 0 and mk(T[a]):
            a = T[a]["parent"]
        if a < 0:
            C.append(i)
    if len(C) > max_c or any(T[v]["depth"] > max_d for v in C):
        return None
    code, sm = {}, {}
    for v in C:
        c, m, w, s = 0, ck(T[v]), v, {}
        s[T[v]["depth"]] = m
        while T[w]["parent"] >= 0:
            a = T[w]["parent"]
            if T[a]["kid1"] == w:
                c |= 1 << (31 - T[a]["depth"])
            m = min(m, ck(T[a]))
            s[T[a]["depth"]] = m
            w = a
        code[v], sm[v] = c, s
    rank = {}
    for v in C:
        dv, before = T[v]["depth"], 0
        for u in C:
            if u == v:
                continue
            if ck(T[u]) == ck(T[v]):
                return None
            if not mk(T[u]):
                continue
            du = T[u]["depth"]
            x = code[u] ^ code[v]
            lca = min(32 - x.bit_length(), du, dv)
            if lca == du:
                before += 1
            elif lca != dv:
                before += sm[u][lca + 1] > sm[v][lca + 1]
        if not T[v]["expanded"] and before < K:
            return None
        if mk(T[v]) and before < K:
            rank[v] = before
    out, alg = {}, T[0]["local"]
    for v, r in rank.items():
        p = T[v]["parent"]
        cur = 0 if p < 0 else (1 if T[p]["kid0"] == v else 2) + 2 * rank[p]
        out[cur] = ("split", v, 1 + 2 * r, 2 + 2 * r)
        for kid, tid in ((T[v]["kid0"], 1 + 2 * r), (T[v]["kid1"], 2 + 2 * r)):
            if kid not in rank:
                out[tid] = ("leaf", kid)
        if T[v]["depth"] + 1 < max_depth:
            k0, k1 = T[v]["kid0"], T[v]["kid1"]
            alg += T[k0 if T[k0]["n"] <= T[k1]["n"] else k1]["local"]
    if not rank:
        out[0] = ("leaf", 0)
    return 0, 1 + 2 * len(rank), out, alg


def _random_grown_table(rng, ties, D=None, p_expand=0.9, max_nodes=None, n_root=None):
    """A node table as the level loop leaves it: nodes numbered level by level,
    some expanded nodes, some candidates left unexpanded (pruned), splits with
    no valid feature, rows split unevenly (some under min_samples_leaf)."""
    D = int(rng.integers(2, 9)) if D is None else D
    T = [dict(depth=0, parent=-1, n=int(rng.integers(50, 5000)) if n_root is None else n_root)]
    level = [0]
    while level:
        nxt = []
        for v in level:
            x = T[v]
            x["feat"] = -1 if x["depth"] >= D or rng.random() < 0.08 else int(rng.integers(0, 50))
            g = rng.exponential(1.0) * np.exp(-0.2 * x["depth"]) - 0.05
            x["gain"] = float(np.round(g, 1) if ties else g)
            x["local"] = int(x["n"] * rng.random())
            x["expanded"] = int(x["feat"] >= 0 and rng.random() < p_expand and
                                (max_nodes is None or len(T) + 2 <= max_nodes))
            x["kid0"] = x["kid1"] = -1
        for v in level:
            x = T[v]
            if not x["expanded"]:
                continue
            n0 = int(rng.binomial(x["n"], rng.uniform(0.02, 0.98)))
            x["kid0"], x["kid1"] = len(T), len(T) + 1
            T.append(dict(depth=x["depth"] + 1, parent=v, n=n0))
            T.append(dict(depth=x["depth"] + 1, parent=v, n=x["n"] - n0))
            nxt += [x["kid0"], x["kid1"]]
        level = nxt
    return T, D


def test_ranked_replay_matches_the_loop():
    """The ranked replay gives the loop's tree (node numbering, leaves, rows
    counted) whenever it does not hand over, and hands over only on equal keys
    or an unexpanded candidate the loop reaches (where the loop reports
    status 1)."""
    rng = np.random.default_rng(11)
    fast = handed = 0
    for case in range(1500):
        ties = case % 3 == 0
        T, D = _random_grown_table(rng, ties)
        max_leaves = int(rng.integers(1, 70))
        gamma = float(rng.choice([0.0, 0.0, 0.3, -1.0]))
        msl = int(rng.choice([1, 20, 200]))
        max_depth = D + int(rng.integers(0, 2))
        loop = _replay_loop(T, max_leaves, gamma, msl, max_depth)
        ranked = _replay_ranked(T, max_leaves, gamma, msl, max_depth)
        if ranked is None:
            handed += 1
            continue
        assert loop[0] == 0, case    # the loop would have reached an unexpanded node
        fast += 1
        assert loop == ranked, case
    assert fast > 800 and handed > 50, (fast, handed)


def _compact_rows_restated(mask, tile=4096, per=16):
    """k_compact_rows' index arithmetic: tiles of `tile` mask bytes, thread t
    of a tile takes bytes 16 t .. 16 t + 15 (a 16-byte load, or byte loads
    past the end), a block exclusive scan of the threads' in-bag counts, the
    tiles' offsets from their predecessors' totals (the look-back), and each
    thread's rows written in order from offset + its scan value."""
    n = len(mask)
    out = np.full(n, -1, np.int64)
    total = 0
    for t0 in range(0, n, tile):
        counts, bits = [], []
        for th in range(tile // per):
            base = t0 + per * th
            b = [k for k in range(per) if base + k < n and mask[base + k] != 0]
            bits.append(b)
            counts.append(len(b))
        excl = np.concatenate([[0], np.cumsum(counts)[:-1]])
        off = total   # the look-back: the sum of the earlier tiles' counts
        for th, b in enumerate(bits):
            o = off + int(excl[th])
            for k in b:
                assert out[o] == -1
                out[o] = t0 + per * th + k
                o += 1
        total += int(sum(counts))
    return out[:total], total


@pytest.mark.parametrize("n", [1, 15, 16, 17, 4095, 4096, 4097, 20_003])
@pytest.mark.parametrize("fill", ["random", "none", "all"])
def test_compact_rows_index_arithmetic(n, fill):
    """The one-pass compaction gives the in-bag rows in ascending order and
    their count, for ragged tails, empty and full masks."""
    rng = np.random.default_rng(n)
    mask = {"random": (rng.random(n) < 0.75), "none": np.zeros(n, bool), "all": np.ones(n, bool)}[fill]
    mask = mask.astype(np.uint8) * rng.integers(1, 255, n).astype(np.uint8)   # any nonzero byte is in bag
    rows, total = _compact_rows_restated(mask)
    want = np.flatnonzero(mask)
    assert total == len(want)
    assert np.array_equal(rows, want)



def test_ranked_replay_at_its_size_limits():
    """Deep tables (depth 10-17, up to 2048 nodes): the ranked form matches the
    loop wherever it does not hand over, and it hands over on every table with
    a candidate deeper than 15 or more than 256 candidates."""
    rng = np.random.default_rng(29)
    over = fast = 0
    for case in range(40):
        D = int(rng.integers(10, 18))
        T, D = _random_grown_table(rng, ties=False, D=D, p_expand=0.85, max_nodes=2048, n_root=1_000_000)
        max_leaves = int(rng.integers(20, 128))
        loop = _replay_loop(T, max_leaves, 0.0, 1, D + 1)
        ranked = _replay_ranked(T, max_leaves, 0.0, 1, D + 1)
        # the candidates: key > 0 and every ancestor a makeable split
        mk = lambda x: (x["feat"] >= 0 and x["gain"] > 0.0 and x["expanded"] and T[x["kid0"]]["n"] >= 1 and
                        T[x["kid1"]]["n"] >= 1)
        cands = []
        for i, x in enumerate(T):
            if not (x["feat"] >= 0 and x["gain"] > 0.0):
                continue
            a = x["parent"]
            while a >= 0 and mk(T[a]):
                a = T[a]["parent"]
            if a < 0:
                cands.append(i)
        beyond = len(cands) > 256 or any(T[v]["depth"] > 15 for v in cands)
        if beyond:
            assert ranked is None, case
            over += 1
        elif ranked is not None:
            fast += 1
            assert loop == ranked, case
    assert fast > 0 and over > 0, (fast, over)
