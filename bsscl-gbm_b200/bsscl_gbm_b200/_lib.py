"""ctypes binding of libgbm_b200.so (the C ABI declared in include/gbm_b200.h).

The library is the only compute path of this package: importing works
without a GPU, but every engine call fails loudly (RuntimeError) when the
shared object is missing or no CUDA device is present.  There is no CPU
fallback.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgbm_b200.so")
CSRC = os.path.join(os.path.dirname(HERE), "csrc")

GBM_OK = 0
ERRORS = {1: "invalid argument", 2: "allocation failed", 3: "CUDA error", 4: "bad state",
          5: "communicator error", 6: "timeout", 7: "unsupported"}

# Every symbol include/gbm_b200.h declares.
EXPORTS = (
    "gbm_ctx_create", "gbm_ctx_destroy", "gbm_last_error", "gbm_ctx_init_comm",
    "gbm_nccl_unique_id", "gbm_upload_bins", "gbm_upload_labels", "gbm_round", "gbm_build_tree",
    "gbm_scale_bits", "gbm_get_F", "gbm_get_grad", "gbm_predict", "gbm_predict_set_model",
    "gbm_predict_upload", "gbm_predict_run", "gbm_predict_fetch", "gbm_sync",
    "gbm_sampler_create", "gbm_sampler_next", "gbm_sampler_destroy", "gbm_sampler_next_rows",
    "gbm_sampler_n_sub", "gbm_sampler_n_feat", "gbm_round_sampled",
    "gbm_set_profiling", "gbm_get_stats", "gbm_reset_stats", "gbm_event_record",
    "gbm_event_elapsed", "gbm_predict_noalloc", "gbm_fit_rounds", "gbm_upload_bins_u16",
    "gbm_set_l2_flush", "gbm_bin_edges", "gbm_upload_binned_rows", "gbm_bin_features",
    "gbm_predict_upload_raw", "gbm_predict_raw", "gbm_test_peer_wait", "gbm_upload_labels_mc",
    "gbm_round_mc", "gbm_get_F_mc", "gbm_get_grad_mc", "gbm_upload_targets", "gbm_round_reg",
    "gbm_check_model", "gbm_sampler_create_device", "gbm_predict_upload_u16", "gbm_round_mc_sampled",
    "gbm_round_reg_sampled",
)


class GbmParams(C.Structure):
    _fields_ = [("reg_lambda", C.c_double), ("gamma", C.c_double),
                ("min_child_weight", C.c_double), ("learning_rate", C.c_double),
                ("min_samples_leaf", C.c_int32), ("max_depth", C.c_int32),
                ("max_leaves", C.c_int32), ("grow_policy", C.c_int32),
                ("monotone", C.c_void_p), ("nan_direction", C.c_int32), ("nan_bin_id", C.c_void_p)]


def with_nan_direction(params, nan_bin_id):
    """params learning the NaN direction (gbm_params.nan_direction) for the
    features whose nan_bin_id is 0; returns (params, the int32 array params
    points at, which the caller keeps alive while params is used)."""
    nb = np.ascontiguousarray(nan_bin_id, dtype=np.int32)
    params.nan_direction = 1
    params.nan_bin_id = nb.ctypes.data_as(C.c_void_p)
    return params, nb


class GbmTreeOut(C.Structure):
    _fields_ = [("capacity", C.c_int32), ("tf", C.c_void_p), ("tt", C.c_void_p),
                ("tv", C.c_void_p), ("tl", C.c_void_p), ("tr", C.c_void_p),
                ("sg", C.c_void_p), ("n_nodes", C.c_int32), ("leaf_of_row", C.c_void_p),
                ("nan_right", C.c_void_p)]


class GbmPacked(C.Structure):
    _fields_ = [("features", C.c_void_p), ("thresholds", C.c_void_p), ("values", C.c_void_p),
                ("left", C.c_void_p), ("right", C.c_void_p), ("offsets", C.c_void_p),
                ("n_trees", C.c_int32), ("nan_right", C.c_void_p)]


class GbmStats(C.Structure):
    _fields_ = [("kernel_launches", C.c_int64), ("hist_launches", C.c_int64),
                ("hist_rows", C.c_int64), ("waves", C.c_int64), ("hist_ms", C.c_double),
                ("hist_alg_bytes", C.c_double), ("host_sample_ms", C.c_double),
                ("host_sync_ms", C.c_double), ("host_replay_ms", C.c_double),
                ("flush_ms", C.c_double), ("hist_updates", C.c_double),
                ("host_comm_ms", C.c_double), ("comm_ms", C.c_double), ("comm_bytes", C.c_double),
                ("peer_wait_ms", C.c_double), ("sampler_ms", C.c_double),
                ("sampler_stall_ms", C.c_double)]


_lib = None


def build(force=False):
    """Compile libgbm_b200.so for sm_100a with nvcc (see csrc/Makefile)."""
    import subprocess
    if force and os.path.exists(LIB_PATH):
        os.remove(LIB_PATH)
    subprocess.run(["make", "-s", "-C", CSRC], check=True)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"libgbm_b200.so not found at {LIB_PATH}; build it with "
            "`make -C bsscl-gbm_b200/csrc` (nvcc, sm_100a). There is no CPU fallback.")
    L = C.CDLL(LIB_PATH)
    P, i32, i64, f64 = C.c_void_p, C.c_int32, C.c_int64, C.c_double
    L.gbm_ctx_create.argtypes = [i32, C.POINTER(C.c_void_p)]
    L.gbm_ctx_destroy.argtypes = [P]
    L.gbm_ctx_destroy.restype = None
    L.gbm_last_error.argtypes = [P]
    L.gbm_last_error.restype = C.c_char_p
    L.gbm_ctx_init_comm.argtypes = [P, P, i32, i32, i32]
    L.gbm_nccl_unique_id.argtypes = [P]
    L.gbm_upload_bins.argtypes = [P, P, i64, i32, P]
    L.gbm_upload_labels.argtypes = [P, P, P, f64, i64]
    L.gbm_round.argtypes = [P, P, P, i32, C.POINTER(GbmParams), C.POINTER(GbmTreeOut),
                            C.POINTER(C.c_double)]
    L.gbm_build_tree.argtypes = [P, P, P, P, P, i32, C.POINTER(GbmParams), C.POINTER(GbmTreeOut)]
    L.gbm_scale_bits.argtypes = [P]
    L.gbm_scale_bits.restype = i32
    L.gbm_get_F.argtypes = [P, P]
    L.gbm_get_grad.argtypes = [P, P, P]
    L.gbm_predict.argtypes = [P, P, i64, i32, C.POINTER(GbmPacked), f64, f64, P, P]
    L.gbm_predict_set_model.argtypes = [P, C.POINTER(GbmPacked), i32]
    L.gbm_predict_upload.argtypes = [P, P, i64, i32]
    L.gbm_predict_upload_u16.argtypes = [P, P, i64, i32]
    L.gbm_predict_run.argtypes = [P, f64, f64]
    L.gbm_predict_fetch.argtypes = [P, P, P]
    L.gbm_sync.argtypes = [P]
    L.gbm_sampler_create_device.argtypes = [C.c_uint32, i64, i32, f64, i32, i32, i32, C.POINTER(C.c_void_p)]
    L.gbm_sampler_create.argtypes = [C.c_uint32, i64, i32, i64, i32, i32, i32, i32,
                                     C.POINTER(C.c_void_p)]
    L.gbm_sampler_next.argtypes = [P, P, P, P]
    L.gbm_sampler_next_rows.argtypes = [P, P, P]
    L.gbm_sampler_n_sub.argtypes = [P]
    L.gbm_sampler_n_sub.restype = i64
    L.gbm_sampler_n_feat.argtypes = [P]
    L.gbm_sampler_n_feat.restype = i32
    L.gbm_round_sampled.argtypes = [P, P, i64, C.POINTER(GbmParams), C.POINTER(GbmTreeOut),
                                    C.POINTER(C.c_double)]
    L.gbm_upload_bins_u16.argtypes = [P, P, i64, i32, P]
    L.gbm_set_l2_flush.argtypes = [P, i64]
    L.gbm_fit_rounds.argtypes = [P, P, i64, C.POINTER(GbmParams), i32, C.POINTER(GbmTreeOut),
                                 P]
    L.gbm_sampler_destroy.argtypes = [P]
    L.gbm_sampler_destroy.restype = None
    L.gbm_set_profiling.argtypes = [P, i32]
    L.gbm_get_stats.argtypes = [P, C.POINTER(GbmStats)]
    L.gbm_reset_stats.argtypes = [P]
    L.gbm_event_record.argtypes = [P, i32]
    L.gbm_event_elapsed.argtypes = [P, i32, i32, C.POINTER(C.c_float)]
    L.gbm_bin_edges.argtypes = [P, P, i64, i32, i32, i32, P, P, i32, P, P, P]
    L.gbm_upload_binned_rows.argtypes = [P, i64, i64, P, i32, P, P]
    L.gbm_bin_features.argtypes = [P, P, i64, i32, i32, P, i32, P, P, P]
    L.gbm_predict_upload_raw.argtypes = [P, P, i64, i32, i32, P, i32, P, P]
    L.gbm_predict_raw.argtypes = [P, P, i64, i32, i32, P, i32, P, P, C.POINTER(GbmPacked), f64,
                                  f64, P, P]
    L.gbm_test_peer_wait.argtypes = [i32, i32]
    L.gbm_upload_labels_mc.argtypes = [P, P, i32, P, i64]
    L.gbm_round_mc.argtypes = [P, P, P, i32, C.POINTER(GbmParams), C.POINTER(GbmTreeOut), C.POINTER(C.c_double)]
    L.gbm_round_mc_sampled.argtypes = [P, P, i64, C.POINTER(GbmParams), C.POINTER(GbmTreeOut),
                                       C.POINTER(C.c_double)]
    L.gbm_round_reg_sampled.argtypes = [P, P, i64, C.POINTER(GbmParams), C.POINTER(GbmTreeOut),
                                        C.POINTER(C.c_double)]
    L.gbm_get_F_mc.argtypes = [P, P]
    L.gbm_get_grad_mc.argtypes = [P, i32, P, P]
    L.gbm_upload_targets.argtypes = [P, P, f64, i32, i64]
    L.gbm_round_reg.argtypes = [P, P, P, i32, C.POINTER(GbmParams), C.POINTER(GbmTreeOut), C.POINTER(C.c_double)]
    L.gbm_predict_noalloc.argtypes = [P, i64, i32, P, P, P, P, P, P, i32, i32, f64, f64, P, P, P,
                                      C.c_char_p, i32]
    L.gbm_check_model.argtypes = [C.POINTER(GbmPacked), i32, C.c_char_p, i32]
    _lib = L
    return L


def ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _tree(tf, tt, tv, tl, tr, nc, sg, nan_right=None):
    """A tree in the reference's tuple layout (tf, tt, tv, tl, tr, nc, sg),
    with the per-node NaN direction appended when the round learned it."""
    t = (tf, tt, tv, tl, tr, int(nc), sg)
    return t if nan_right is None else t + (nan_right,)


def check_model(packed, n_trees, n_features):
    """Host-side checks of a packed ensemble (gbm_check_model): raises
    ValueError with the library's message when a walk could leave its tree
    (offsets not starting at 0 or not increasing, a child not after its
    parent or outside its tree, a feature >= n_features, a negative
    threshold).  Needs no GPU."""
    L = lib()
    s, keep = Engine.packed_struct(packed, n_trees)
    buf = C.create_string_buffer(256)
    rc = L.gbm_check_model(C.byref(s), int(n_features), buf, 256)
    if rc != GBM_OK:
        raise ValueError(f"gbm_check_model: {buf.value.decode()} ({ERRORS.get(rc, rc)})")


class Engine:
    """One device context (one GPU, one CUDA stream)."""

    def __init__(self, device=0):
        self._L = lib()
        self._h = C.c_void_p()
        rc = self._L.gbm_ctx_create(int(device), C.byref(self._h))
        if rc != GBM_OK:
            msg = self.last_error()
            self.close()
            raise RuntimeError(f"gbm_ctx_create(device={device}) failed: {msg}")

    # -- plumbing --
    def last_error(self):
        if not self._h:
            return "no context"
        return self._L.gbm_last_error(self._h).decode(errors="replace")

    def check(self, rc, what):
        if rc != GBM_OK:
            raise RuntimeError(f"{what} failed ({ERRORS.get(rc, rc)}): {self.last_error()}")

    def close(self):
        if getattr(self, "_h", None):
            self._L.gbm_ctx_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- multi-GPU --
    @staticmethod
    def nccl_unique_id():
        buf = (C.c_uint8 * 128)()
        rc = lib().gbm_nccl_unique_id(C.cast(buf, C.c_void_p))
        if rc != GBM_OK:
            raise RuntimeError("ncclGetUniqueId failed (is libnccl.so.2 available?)")
        return bytes(buf)

    def init_comm(self, uid: bytes, nranks: int, rank: int, timeout_ms: int = 60000):
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        self.check(self._L.gbm_ctx_init_comm(self._h, C.cast(buf, C.c_void_p), nranks, rank,
                                             timeout_ms), "gbm_ctx_init_comm")
        self._comm_world = (nranks, rank)

    # -- training --
    def upload_bins(self, xbin, counts):
        """Bins [n][p] as uint8 (gbm_upload_bins) or the reference's uint16
        (gbm_upload_bins_u16, narrowed on the device)."""
        cnt = np.ascontiguousarray(counts, dtype=np.int32)
        if np.asarray(xbin).dtype == np.uint16:
            xb = np.ascontiguousarray(xbin)
            n, p = xb.shape
            rc = self._L.gbm_upload_bins_u16(self._h, ptr(xb), n, p, ptr(cnt))
        else:
            xb = np.ascontiguousarray(xbin, dtype=np.uint8)
            n, p = xb.shape
            rc = self._L.gbm_upload_bins(self._h, ptr(xb), n, p, ptr(cnt))
        self.n, self.p = n, p
        self.check(rc, "gbm_upload_bins")

    # -- binning on the device --
    @staticmethod
    def _raw(X):
        """(contiguous float32/float64 matrix, dtype code) of a raw matrix."""
        X = np.asarray(X)
        if X.dtype != np.float32:
            X = np.asarray(X, dtype=np.float64)
        return np.ascontiguousarray(X), (0 if X.dtype == np.float32 else 1)

    @staticmethod
    def _tables(edges, counts, nan_bin):
        e = np.ascontiguousarray(edges, dtype=np.float64)
        return (e, np.ascontiguousarray(counts, dtype=np.int32),
                np.ascontiguousarray(nan_bin, dtype=np.int32))

    def bin_edges(self, X, n_bins, categorical=None):
        """``_build_bin_edges`` (sample_weight=None) on the GPU:
        ``(edges_2d [p, max_b] float64, counts int32 [p], nan_bin_id int32 [p])``.
        The matrix stays on the device for :meth:`upload_binned_rows`."""
        Xc, dt = self._raw(X)
        n, p = Xc.shape
        stride = max(int(n_bins) + 2, 65)
        edges = np.empty((p, stride), np.float64)
        counts = np.empty(p, np.int32)
        nanb = np.empty(p, np.int32)
        maxb = C.c_int32(0)
        cat = None
        if categorical is not None:
            cat = np.zeros(p, np.uint8)
            cat[list(categorical)] = 1
        self.check(self._L.gbm_bin_edges(self._h, ptr(Xc), n, p, dt, int(n_bins), ptr(cat), ptr(edges),
                                         stride, ptr(counts), ptr(nanb), C.byref(maxb)),
                   "gbm_bin_edges")
        self._binned = (n, p)
        return np.ascontiguousarray(edges[:, :maxb.value]), counts, nanb

    def upload_binned_rows(self, lo, hi, edges, counts, nan_bin):
        """Training bins from rows [lo, hi) of the matrix given to :meth:`bin_edges`."""
        e, cnt, nb = self._tables(edges, counts, nan_bin)
        self.check(self._L.gbm_upload_binned_rows(self._h, int(lo), int(hi), ptr(e), e.shape[1],
                                                  ptr(cnt), ptr(nb)), "gbm_upload_binned_rows")
        self.n, self.p = hi - lo, e.shape[0]

    def bin_features(self, X, edges, counts, nan_bin):
        """The reference's raw bin ids (``_bin_features``), uint16 [n, p], computed on the GPU."""
        Xc, dt = self._raw(X)
        n, p = Xc.shape
        e, cnt, nb = self._tables(edges, counts, nan_bin)
        out = np.empty((n, p), np.uint16)
        self.check(self._L.gbm_bin_features(self._h, ptr(Xc), n, p, dt, ptr(e), e.shape[1], ptr(cnt),
                                            ptr(nb), ptr(out)), "gbm_bin_features")
        return out

    def predict_raw(self, X, edges, counts, nan_bin, packed, n_trees, lr, base, want_F=True,
                    want_proba=True):
        """Predict from a raw matrix: binned on the GPU, then the ensemble."""
        Xc, dt = self._raw(X)
        n, p = Xc.shape
        e, cnt, nb = self._tables(edges, counts, nan_bin)
        s, keep = self.packed_struct(packed, n_trees)
        F = np.empty(n, np.float64) if want_F else None
        P = np.empty(n, np.float64) if want_proba else None
        self.check(self._L.gbm_predict_raw(self._h, ptr(Xc), n, p, dt, ptr(e), e.shape[1], ptr(cnt),
                                           ptr(nb), C.byref(s), float(lr), float(base), ptr(F),
                                           ptr(P)), "gbm_predict_raw")
        return F, P

    def predict_upload_raw(self, X, edges, counts, nan_bin):
        Xc, dt = self._raw(X)
        e, cnt, nb = self._tables(edges, counts, nan_bin)
        self._pn = Xc.shape[0]
        self.check(self._L.gbm_predict_upload_raw(self._h, ptr(Xc), Xc.shape[0], Xc.shape[1], dt,
                                                  ptr(e), e.shape[1], ptr(cnt), ptr(nb)),
                   "gbm_predict_upload_raw")

    def set_l2_flush(self, nbytes):
        """Benchmark aid: evict L2 at the start of every round (0 = off)."""
        self.check(self._L.gbm_set_l2_flush(self._h, int(nbytes)), "gbm_set_l2_flush")

    def upload_labels(self, y01, w2, base_score, n_global=0):
        y = np.ascontiguousarray(y01, dtype=np.uint8)
        w = np.ascontiguousarray(w2, dtype=np.float64)
        self.check(self._L.gbm_upload_labels(self._h, ptr(y), ptr(w), float(base_score),
                                             int(n_global)), "gbm_upload_labels")

    def round(self, inbag_mask, feat_idx, params: GbmParams, capacity, want_leaf=False):
        mask = np.ascontiguousarray(inbag_mask, dtype=np.uint8)
        fidx = np.ascontiguousarray(feat_idx, dtype=np.int32)
        tf = np.empty(capacity, np.int32); tt = np.empty(capacity, np.int64)
        tv = np.empty(capacity, np.float64); tl = np.empty(capacity, np.int32)
        tr = np.empty(capacity, np.int32); sg = np.empty(capacity, np.float64)
        leaf = np.empty(self.n, np.int32) if want_leaf else None
        nr = np.empty(capacity, np.int32) if params.nan_direction else None
        out = GbmTreeOut(capacity, ptr(tf), ptr(tt), ptr(tv), ptr(tl), ptr(tr), ptr(sg), 0,
                         ptr(leaf), ptr(nr))
        loss = C.c_double(0.0)
        self.check(self._L.gbm_round(self._h, ptr(mask), ptr(fidx), len(fidx), C.byref(params),
                                     C.byref(out), C.byref(loss)), "gbm_round")
        return _tree(tf, tt, tv, tl, tr, out.n_nodes, sg, nr), float(loss.value), leaf

    # -- regression --
    def upload_targets(self, y, init_score, loss="mse", n_global=0):
        yy = np.ascontiguousarray(y, dtype=np.float64)
        self.check(self._L.gbm_upload_targets(self._h, ptr(yy), float(init_score), 0 if loss == "mse" else 1,
                                              int(n_global)), "gbm_upload_targets")

    def round_reg(self, inbag_mask, feat_idx, params: GbmParams, capacity, want_leaf=False):
        mask = np.ascontiguousarray(inbag_mask, dtype=np.uint8)
        fidx = np.ascontiguousarray(feat_idx, dtype=np.int32)
        tf = np.empty(capacity, np.int32); tt = np.empty(capacity, np.int64)
        tv = np.empty(capacity, np.float64); tl = np.empty(capacity, np.int32)
        tr = np.empty(capacity, np.int32); sg = np.empty(capacity, np.float64)
        leaf = np.empty(self.n, np.int32) if want_leaf else None
        out = GbmTreeOut(capacity, ptr(tf), ptr(tt), ptr(tv), ptr(tl), ptr(tr), ptr(sg), 0, ptr(leaf))
        loss = C.c_double(0.0)
        self.check(self._L.gbm_round_reg(self._h, ptr(mask), ptr(fidx), len(fidx), C.byref(params),
                                         C.byref(out), C.byref(loss)), "gbm_round_reg")
        return (tf, tt, tv, tl, tr, int(out.n_nodes), sg), float(loss.value), leaf

    def round_reg_sampled(self, sampler, row_offset, params: GbmParams, capacity):
        """gbm_round_reg_sampled: the tree with the round's subsample drawn by
        `sampler` (its shuffle applied on the device) and the train loss."""
        tf = np.empty(capacity, np.int32); tt = np.empty(capacity, np.int64)
        tv = np.empty(capacity, np.float64); tl = np.empty(capacity, np.int32)
        tr = np.empty(capacity, np.int32); sg = np.empty(capacity, np.float64)
        out = GbmTreeOut(capacity, ptr(tf), ptr(tt), ptr(tv), ptr(tl), ptr(tr), ptr(sg), 0, None)
        loss = C.c_double(0.0)
        self.check(self._L.gbm_round_reg_sampled(self._h, sampler._h, int(row_offset), C.byref(params),
                                                 C.byref(out), C.byref(loss)), "gbm_round_reg_sampled")
        return (tf, tt, tv, tl, tr, int(out.n_nodes), sg), float(loss.value)

    # -- multi-class softmax --
    def upload_labels_mc(self, y, n_classes, class_w, n_global=0):
        yy = np.ascontiguousarray(y, dtype=np.uint8)
        w = np.ascontiguousarray(class_w, dtype=np.float64)
        self.K = int(n_classes)
        self.check(self._L.gbm_upload_labels_mc(self._h, ptr(yy), self.K, ptr(w), int(n_global)),
                   "gbm_upload_labels_mc")

    def round_mc(self, inbag_mask, feat_idx, params: GbmParams, capacity, want_leaf=False):
        """gbm_round_mc: K trees (one per class) and the round's train loss."""
        mask = np.ascontiguousarray(inbag_mask, dtype=np.uint8)
        fidx = np.ascontiguousarray(feat_idx, dtype=np.int32)
        K = self.K
        arrs, leaves = [], []
        outs = (GbmTreeOut * K)()
        for k in range(K):
            a = (np.empty(capacity, np.int32), np.empty(capacity, np.int64), np.empty(capacity, np.float64),
                 np.empty(capacity, np.int32), np.empty(capacity, np.int32), np.empty(capacity, np.float64))
            leaf = np.empty(self.n, np.int32) if want_leaf else None
            arrs.append(a)
            leaves.append(leaf)
            outs[k] = GbmTreeOut(capacity, ptr(a[0]), ptr(a[1]), ptr(a[2]), ptr(a[3]), ptr(a[4]),
                                 ptr(a[5]), 0, ptr(leaf))
        loss = C.c_double(0.0)
        self.check(self._L.gbm_round_mc(self._h, ptr(mask), ptr(fidx), len(fidx), C.byref(params), outs,
                                        C.byref(loss)), "gbm_round_mc")
        trees = [(a[0], a[1], a[2], a[3], a[4], int(outs[k].n_nodes), a[5]) for k, a in enumerate(arrs)]
        return trees, float(loss.value), leaves

    def round_mc_sampled(self, sampler, row_offset, params: GbmParams, capacity):
        """gbm_round_mc_sampled: K trees with the round's subsample drawn by
        `sampler` (its shuffle applied on the device) and the train loss."""
        K = self.K
        blocks = [np.empty((K, capacity), t) for t in (np.int32, np.int64, np.float64, np.int32, np.int32,
                                                        np.float64)]
        outs = (GbmTreeOut * K)()
        for k in range(K):
            outs[k] = GbmTreeOut(capacity, *(ptr(b[k]) for b in blocks), 0, None)
        loss = C.c_double(0.0)
        self.check(self._L.gbm_round_mc_sampled(self._h, sampler._h, int(row_offset), C.byref(params), outs,
                                                C.byref(loss)), "gbm_round_mc_sampled")
        trees = [(blocks[0][k], blocks[1][k], blocks[2][k], blocks[3][k], blocks[4][k], int(outs[k].n_nodes),
                  blocks[5][k]) for k in range(K)]
        return trees, float(loss.value)

    def get_F_mc(self):
        F = np.empty((self.K, self.n), np.float64)
        self.check(self._L.gbm_get_F_mc(self._h, ptr(F)), "gbm_get_F_mc")
        return F

    def get_grad_mc(self, k):
        g = np.empty(self.n, np.float64)
        h = np.empty(self.n, np.float64)
        self.check(self._L.gbm_get_grad_mc(self._h, int(k), ptr(g), ptr(h)), "gbm_get_grad_mc")
        return g, h

    def round_sampled(self, sampler, row_offset, params: GbmParams, capacity, want_leaf=False):
        """gbm_round with the subsample drawn by `sampler` (global row ids)."""
        tf = np.empty(capacity, np.int32); tt = np.empty(capacity, np.int64)
        tv = np.empty(capacity, np.float64); tl = np.empty(capacity, np.int32)
        tr = np.empty(capacity, np.int32); sg = np.empty(capacity, np.float64)
        leaf = np.empty(self.n, np.int32) if want_leaf else None
        nr = np.empty(capacity, np.int32) if params.nan_direction else None
        out = GbmTreeOut(capacity, ptr(tf), ptr(tt), ptr(tv), ptr(tl), ptr(tr), ptr(sg), 0,
                         ptr(leaf), ptr(nr))
        loss = C.c_double(0.0)
        self.check(self._L.gbm_round_sampled(self._h, sampler._h, int(row_offset), C.byref(params),
                                             C.byref(out), C.byref(loss)), "gbm_round_sampled")
        return _tree(tf, tt, tv, tl, tr, out.n_nodes, sg, nr), float(loss.value), leaf

    def fit_rounds(self, sampler, row_offset, params: GbmParams, capacity, n_rounds):
        """n_rounds rounds queued back to back (gbm_fit_rounds): a list of
        (tree, train_loss), the same as n_rounds round_sampled calls."""
        n_rounds = int(n_rounds)
        R = max(1, n_rounds)
        # one block per field, a row per round (few allocations for long fits)
        blocks = (np.empty((R, capacity), np.int32), np.empty((R, capacity), np.int64),
                  np.empty((R, capacity), np.float64), np.empty((R, capacity), np.int32),
                  np.empty((R, capacity), np.int32), np.empty((R, capacity), np.float64),
                  np.empty((R, capacity), np.int32) if params.nan_direction else None)
        arrays = [tuple(b[r] if b is not None else None for b in blocks) for r in range(n_rounds)]
        outs = (GbmTreeOut * R)()
        for r in range(n_rounds):
            a = arrays[r]
            outs[r] = GbmTreeOut(capacity, ptr(a[0]), ptr(a[1]), ptr(a[2]), ptr(a[3]), ptr(a[4]),
                                 ptr(a[5]), 0, None, ptr(a[6]))
        losses = np.zeros(max(1, n_rounds), np.float64)
        self.check(self._L.gbm_fit_rounds(self._h, sampler._h, int(row_offset), C.byref(params),
                                          n_rounds, outs, ptr(losses)), "gbm_fit_rounds")
        res = []
        for r in range(n_rounds):
            tf, tt, tv, tl, tr, sg, nr = arrays[r]
            res.append((_tree(tf, tt, tv, tl, tr, outs[r].n_nodes, sg, nr), float(losses[r])))
        return res

    def build_tree(self, grad, hess, inbag_mask, feat_idx, params: GbmParams, capacity):
        """One tree from given gradients (the reference's _build_one_tree seam)."""
        g = np.ascontiguousarray(grad, dtype=np.float64)
        h = np.ascontiguousarray(hess, dtype=np.float64)
        mask = np.ascontiguousarray(inbag_mask, dtype=np.uint8)
        fidx = np.ascontiguousarray(feat_idx, dtype=np.int32)
        tf = np.empty(capacity, np.int32); tt = np.empty(capacity, np.int64)
        tv = np.empty(capacity, np.float64); tl = np.empty(capacity, np.int32)
        tr = np.empty(capacity, np.int32); sg = np.empty(capacity, np.float64)
        nr = np.empty(capacity, np.int32) if params.nan_direction else None
        out = GbmTreeOut(capacity, ptr(tf), ptr(tt), ptr(tv), ptr(tl), ptr(tr), ptr(sg), 0, None, ptr(nr))
        self.check(self._L.gbm_build_tree(self._h, ptr(g), ptr(h), ptr(mask), ptr(fidx), len(fidx),
                                          C.byref(params), C.byref(out)), "gbm_build_tree")
        return _tree(tf, tt, tv, tl, tr, out.n_nodes, sg, nr)

    def scale_bits(self):
        return int(self._L.gbm_scale_bits(self._h))

    def get_F(self):
        F = np.empty(self.n, np.float64)
        self.check(self._L.gbm_get_F(self._h, ptr(F)), "gbm_get_F")
        return F

    def get_grad(self):
        g = np.empty(self.n, np.float64); h = np.empty(self.n, np.float64)
        self.check(self._L.gbm_get_grad(self._h, ptr(g), ptr(h)), "gbm_get_grad")
        return g, h

    # -- predict --
    @staticmethod
    def packed_struct(packed, n_trees):
        keep = {
            "features": np.ascontiguousarray(packed["features"], dtype=np.int16),
            "thresholds": np.ascontiguousarray(packed["thresholds"], dtype=np.int64),
            "values": np.ascontiguousarray(packed["values"], dtype=np.float64),
            "left": np.ascontiguousarray(packed["left"], dtype=np.int32),
            "right": np.ascontiguousarray(packed["right"], dtype=np.int32),
            "offsets": np.ascontiguousarray(packed["offsets"], dtype=np.int32),
        }
        if packed.get("nan_right") is not None:
            keep["nan_right"] = np.ascontiguousarray(packed["nan_right"], dtype=np.uint8)
        s = GbmPacked(ptr(keep["features"]), ptr(keep["thresholds"]), ptr(keep["values"]),
                      ptr(keep["left"]), ptr(keep["right"]), ptr(keep["offsets"]), int(n_trees),
                      ptr(keep.get("nan_right")))
        return s, keep

    def predict(self, xbin, packed, n_trees, lr, base, want_F=True, want_proba=True):
        """gbm_predict on uint8 bins; the reference's uint16 bins (ids up to
        256: 257-bin features) go through gbm_predict_upload_u16."""
        if np.asarray(xbin).dtype == np.uint16:
            xb = np.ascontiguousarray(xbin)
            self.predict_set_model(packed, n_trees, xb.shape[1])
            self.predict_upload(xb)
            self.predict_run(lr, base)
            return self.predict_fetch(want_F, want_proba)
        xb = np.ascontiguousarray(xbin, dtype=np.uint8)
        n, p = xb.shape
        s, keep = self.packed_struct(packed, n_trees)
        F = np.empty(n, np.float64) if want_F else None
        P = np.empty(n, np.float64) if want_proba else None
        self.check(self._L.gbm_predict(self._h, ptr(xb), n, p, C.byref(s), float(lr), float(base),
                                       ptr(F), ptr(P)), "gbm_predict")
        return F, P

    def predict_set_model(self, packed, n_trees, n_features):
        s, keep = self.packed_struct(packed, n_trees)
        self.check(self._L.gbm_predict_set_model(self._h, C.byref(s), int(n_features)),
                   "gbm_predict_set_model")

    def predict_upload(self, xbin):
        """uint8 bins (gbm_predict_upload) or the reference's uint16
        (gbm_predict_upload_u16)."""
        if np.asarray(xbin).dtype == np.uint16:
            xb = np.ascontiguousarray(xbin)
            self._pn = xb.shape[0]
            self.check(self._L.gbm_predict_upload_u16(self._h, ptr(xb), xb.shape[0], xb.shape[1]),
                       "gbm_predict_upload_u16")
            return
        xb = np.ascontiguousarray(xbin, dtype=np.uint8)
        self._pn = xb.shape[0]
        self.check(self._L.gbm_predict_upload(self._h, ptr(xb), xb.shape[0], xb.shape[1]),
                   "gbm_predict_upload")

    def predict_run(self, lr, base):
        self.check(self._L.gbm_predict_run(self._h, float(lr), float(base)), "gbm_predict_run")

    def predict_fetch(self, want_F=True, want_proba=True):
        F = np.empty(self._pn, np.float64) if want_F else None
        P = np.empty(self._pn, np.float64) if want_proba else None
        self.check(self._L.gbm_predict_fetch(self._h, ptr(F), ptr(P)), "gbm_predict_fetch")
        return F, P

    def sync(self):
        self.check(self._L.gbm_sync(self._h), "gbm_sync")

    # -- instrumentation --
    def set_profiling(self, on=True):
        self.check(self._L.gbm_set_profiling(self._h, int(bool(on))), "gbm_set_profiling")

    def stats(self):
        st = GbmStats()
        self.check(self._L.gbm_get_stats(self._h, C.byref(st)), "gbm_get_stats")
        return {k: getattr(st, k) for k, _ in GbmStats._fields_}

    def reset_stats(self):
        self.check(self._L.gbm_reset_stats(self._h), "gbm_reset_stats")

    def event(self, slot):
        self.check(self._L.gbm_event_record(self._h, int(slot)), "gbm_event_record")

    def elapsed_ms(self, a, b):
        ms = C.c_float(0.0)
        self.check(self._L.gbm_event_elapsed(self._h, int(a), int(b), C.byref(ms)),
                   "gbm_event_elapsed")
        return float(ms.value)


class Sampler:
    """The reference's RandomState row/feature subsample stream (native, bit-exact)."""

    def __init__(self, seed, n, p, n_sub, n_feat, subsample_on, colsample_on, look_ahead=2):
        self._L = lib()
        self._h = C.c_void_p()
        self.n, self.p, self.n_sub, self.n_feat = int(n), int(p), int(n_sub), int(n_feat)
        rc = self._L.gbm_sampler_create(C.c_uint32(int(seed) & 0xFFFFFFFF), self.n, self.p,
                                        self.n_sub, self.n_feat, int(bool(subsample_on)),
                                        int(bool(colsample_on)), int(look_ahead),
                                        C.byref(self._h))
        if rc != GBM_OK:
            raise ValueError(f"gbm_sampler_create failed ({ERRORS.get(rc, rc)})")

    @classmethod
    def device(cls, seed, n, p, subsample, n_feat, colsample_on, look_ahead=2):
        """A throughput-mode sampler (gbm_sampler_create_device): features as
        the reference draws them, rows drawn on the device by a counter-based
        hash (each row in-bag with probability `subsample`).  Off the parity
        paths: only the engine's round calls accept it."""
        self = cls.__new__(cls)
        self._L = lib()
        self._h = C.c_void_p()
        self.n, self.p, self.n_feat = int(n), int(p), int(n_feat)
        self.n_sub = max(1, int(self.n * float(subsample)))
        rc = self._L.gbm_sampler_create_device(C.c_uint32(int(seed) & 0xFFFFFFFF), self.n, self.p,
                                               float(subsample), self.n_feat, int(bool(colsample_on)),
                                               int(look_ahead), C.byref(self._h))
        if rc != GBM_OK:
            raise ValueError(f"gbm_sampler_create_device failed ({ERRORS.get(rc, rc)})")
        return self

    def next(self, want_sample=False, want_mask=True):
        s = np.empty(self.n_sub, np.int64) if want_sample else None
        m = np.empty(self.n, np.uint8) if want_mask else None
        f = np.empty(self.n_feat, np.int32)
        rc = self._L.gbm_sampler_next(self._h, ptr(s), ptr(m), ptr(f))
        if rc != GBM_OK:
            raise RuntimeError("gbm_sampler_next failed")
        return s, m, f

    def close(self):
        if getattr(self, "_h", None):
            self._L.gbm_sampler_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
