"""``HybridHistGBMNumbaV1_0_1`` -- the reference's estimator API on the B200 engine.

Mirrors the public surface of src/bsscl_gbm/estimator_v1_0_1.py (E):
constructor and 'auto' resolution (E:1820-1923, E:1925-2029), ``fit``
(E:3070-3271), ``predict_proba`` (E:3274-3336), ``predict`` (E:3345-3368),
``get_params`` / ``set_params`` (E:3773-3796), the fitted attributes
(``trees``, ``_packed_*``, ``_tree_offsets``, ``base_score_``, ``bin_edges``,
``feature_bin_counts``, ``_nan_bin_id``, ``train_loss_history_``,
``val_loss_history_``, ``feature_importances_``, ``times``,
``n_trees_fitted_``) and its ValueErrors.

Every boosting round runs on the GPU through libgbm_b200.so (``gbm_round``);
predict_proba runs ``gbm_predict``.  There is no CPU path: ``device`` must
name a CUDA device ('b200', 'cuda', 'cuda:N'), and a missing device or
library raises.  Objectives: binary log-loss, multi-class softmax and
regression (mse / mae); LambdaRank, focal and custom objectives, GOSS, DART
and categorical features raise NotImplementedError.

Row sharding: when ``torch.distributed`` is initialised with more than one
rank, every rank passes the same full ``X``/``y`` and trains on its
contiguous block of rows; histograms are summed exactly over ranks, so
every rank grows the same trees as one GPU would.
"""

from __future__ import annotations

import os
import time

import numpy as np

from . import binning
from ._lib import Engine, GbmParams, Sampler, with_nan_direction


def _device_index(device):
    if device in ("b200", "cuda", "gpu", "auto"):
        return None
    if isinstance(device, str) and device.startswith("cuda:"):
        return int(device.split(":", 1)[1])
    if isinstance(device, int):
        return device
    raise ValueError(f"device={device!r}: this engine runs on CUDA devices only "
                     "('b200', 'cuda', 'cuda:N'); it has no CPU path")


def _dist():
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            return dist
    except Exception:
        pass
    return None


class HybridHistGBMNumbaV1_0_1:
    """Histogram GBM (binary log-loss) trained and evaluated on NVIDIA B200."""

    def __init__(self, n_estimators='auto', max_depth='auto', learning_rate='auto',
                 n_bins='auto', reg_lambda=1.0, min_samples_leaf=5,
                 min_child_weight='auto', gamma='auto',
                 subsample='auto', colsample_bytree='auto',
                 class_weight='balanced_sqrt',
                 grow_policy='leaf', max_leaves=31, binning_strategy='auto',
                 monotone_constraints=None, categorical_features=None,
                 early_stopping_rounds=None, verbose=True, random_state=None,
                 objective='auto', focal_gamma=2.0, loss='mse', device='b200',
                 sampling_method='uniform', top_rate=0.2, other_rate=0.1,
                 scale_pos_weight=None, custom_objective=None, boosting_type='gbdt',
                 dart_rate=0.1, interaction_constraints=None, nan_direction='left'):
        self.binning_strategy_init = binning_strategy
        self.n_estimators_init = n_estimators
        self.max_depth_init = max_depth
        self.learning_rate_init = learning_rate
        self.n_bins_init = n_bins
        self.reg_lambda = reg_lambda
        self.min_samples_leaf = min_samples_leaf
        self.min_child_weight_init = min_child_weight
        self.gamma_init = gamma
        self.subsample_init = subsample
        self.colsample_init = colsample_bytree
        self.device = device
        _device_index(device)
        self.sampling_method = sampling_method
        self.top_rate = top_rate
        self.other_rate = other_rate
        self.scale_pos_weight = scale_pos_weight
        self.class_weight = class_weight
        self.grow_policy = grow_policy
        self.custom_objective = custom_objective
        self.boosting_type = boosting_type
        self.dart_rate = dart_rate
        self.interaction_constraints = interaction_constraints
        # 'left' (default): the reference's rule, the NaN bin always goes left
        # (E:668).  'learn': every split also weighs sending NaN right and
        # keeps the better direction (no reference counterpart; binary only).
        self.nan_direction = nan_direction
        self.max_leaves = max_leaves
        self.monotone_constraints = monotone_constraints
        self.categorical_features = categorical_features
        self.early_stopping_rounds = early_stopping_rounds
        self.verbose = verbose
        self.random_state = random_state
        self.n_estimators = 100 if n_estimators == 'auto' else n_estimators
        self.max_depth = 5 if max_depth == 'auto' else max_depth
        self.learning_rate = 0.1 if learning_rate == 'auto' else learning_rate
        self.n_bins = 256 if n_bins == 'auto' else n_bins
        self.min_child_weight = 1.0 if min_child_weight == 'auto' else min_child_weight
        self.gamma = 0.0 if gamma == 'auto' else gamma
        self.subsample = 0.8 if subsample == 'auto' else subsample
        self.colsample_bytree = 0.8 if colsample_bytree == 'auto' else colsample_bytree
        self.objective = objective
        self.focal_gamma = focal_gamma
        self.loss = loss
        self.init_score_ = 0.0
        self.trees = []
        self.bin_edges = None
        self.feature_bin_counts = None
        self._max_bins = 0
        self.n_features_in_ = None
        self.n_classes_ = 2
        self.classes_ = None
        self._is_multiclass = False
        self.mc_trees = None
        self.feature_importances_ = None
        self.feature_split_counts_ = None
        self.train_loss_history_ = []
        self.val_loss_history_ = []
        self.n_trees_fitted_ = 0
        self.best_iteration_ = 0
        self.times = {'binning': 0.0, 'training': 0.0, 'inference': 0.0, 'upload': 0.0, 'rounds': 0.0}
        self._packed_features = None
        self._packed_thresholds = None
        self._packed_values = None
        self._packed_left = None
        self._packed_right = None
        self._tree_offsets = None
        self._tree_nan_right = []      # per tree: nan_right [nc] (nan_direction='learn'), else None
        self._packed_nan_right = None
        self._mc_packed = None
        self._nan_bin_id = None
        self._engine = None
        self._engine_dev = None
        self.scale_bits_ = None

    # ------------------------------------------------------------------
    # sklearn-style parameter access (E:3773-3796)
    # ------------------------------------------------------------------
    _PARAM_NAMES = ('n_estimators', 'max_depth', 'learning_rate', 'n_bins', 'reg_lambda',
                    'min_samples_leaf', 'min_child_weight', 'gamma', 'subsample',
                    'colsample_bytree', 'class_weight', 'grow_policy', 'max_leaves',
                    'binning_strategy', 'monotone_constraints', 'categorical_features',
                    'early_stopping_rounds', 'verbose', 'random_state', 'objective',
                    'focal_gamma', 'loss', 'device', 'sampling_method', 'top_rate',
                    'other_rate', 'scale_pos_weight', 'custom_objective', 'boosting_type',
                    'dart_rate', 'interaction_constraints', 'nan_direction')
    _INIT_ALIAS = {'n_estimators': 'n_estimators_init', 'max_depth': 'max_depth_init',
                   'learning_rate': 'learning_rate_init', 'n_bins': 'n_bins_init',
                   'min_child_weight': 'min_child_weight_init', 'gamma': 'gamma_init',
                   'subsample': 'subsample_init', 'colsample_bytree': 'colsample_init',
                   'binning_strategy': 'binning_strategy_init'}

    def get_params(self, deep=True):
        out = {}
        for k in self._PARAM_NAMES:
            out[k] = getattr(self, self._INIT_ALIAS.get(k, k), None)
        return out

    def set_params(self, **params):
        for k, v in params.items():
            if k not in self._PARAM_NAMES:
                raise ValueError(f"Invalid parameter {k!r}")
            if k in self._INIT_ALIAS:
                setattr(self, self._INIT_ALIAS[k], v)
                if v != 'auto':
                    setattr(self, k, v)
            else:
                setattr(self, k, v)
                if k == 'device':
                    _device_index(v)
        return self

    def __getstate__(self):
        st = self.__dict__.copy()
        st['_engine'] = None
        st['_engine_dev'] = None
        return st

    # ------------------------------------------------------------------
    # adaptive hyper-parameters (E:1925-2029)
    # ------------------------------------------------------------------
    def _compute_adaptive_hyperparameters(self, X, y):
        n, p = X.shape
        K = self.n_classes_
        if self.binning_strategy_init == 'auto':
            self.binning_strategy = 'hybrid' if (n > 20000 or p > 40) else 'standard'
        else:
            self.binning_strategy = self.binning_strategy_init
        if self.max_depth_init == 'auto':
            if K > 10:
                self.max_depth = min(8, max(4, int(np.log2(max(n // 8, 8)))))
            else:
                self.max_depth = min(6, max(3, int(np.log2(max(n // 10, 8)))))
        if self.learning_rate_init == 'auto':
            data_std = np.std(X)
            if n > 20000:
                self.learning_rate = 0.08
            elif data_std > 2.0:
                self.learning_rate = 0.10
            elif data_std > 1.5:
                self.learning_rate = 0.12
            elif data_std > 1.0:
                self.learning_rate = 0.15
            elif data_std > 0.5:
                self.learning_rate = 0.18
            else:
                self.learning_rate = 0.20
            if K > 10:
                self.learning_rate *= 0.75
            elif K > 6:
                self.learning_rate *= 0.85
        if self.n_bins_init == 'auto':
            self.n_bins = min(256, p * 8 + 32)
        if self.n_estimators_init == 'auto':
            if K <= 2:
                self.n_estimators = 150
            elif K <= 6:
                self.n_estimators = max(150, min(300, n // 10))
            elif K <= 15:
                self.n_estimators = max(200, min(400, n // 8))
            else:
                self.n_estimators = max(250, min(500, n // 6))
        if self.gamma_init == 'auto':
            self.gamma = 0.0
        if self.min_child_weight_init == 'auto':
            self.min_child_weight = 3.0 if n > 20000 else (2.0 if n > 5000 else 1.0)
        if self.subsample_init == 'auto':
            self.subsample = 0.5 if n > 1000000 else (0.75 if n > 20000 else 0.8)
        if n > 1000000:
            self.reg_lambda = max(self.reg_lambda, 5.0)
        if self.colsample_init == 'auto':
            self.colsample_bytree = 0.7 if p > 40 else 0.8
        if n > 10000:
            self.max_leaves = 63
        elif n < 2000:
            self.max_leaves = 15
        else:
            self.max_leaves = 31
        if self.verbose:
            resolved = {k: getattr(self, k) for k in ('n_estimators', 'max_depth', 'learning_rate', 'n_bins',
                                                      'gamma', 'min_child_weight', 'subsample',
                                                      'colsample_bytree', 'max_leaves', 'reg_lambda')}
            print(f"[bsscl-gbm-b200] {n} x {p}, resolved parameters: {resolved}")

    # ------------------------------------------------------------------
    # class weights and base score (E:2570-2603, E:2829-2835)
    # ------------------------------------------------------------------
    def _class_weight_pair(self, y01):
        if self.scale_pos_weight is not None and self.objective == 'binary':
            return np.array([1.0, float(self.scale_pos_weight)])
        if self.class_weight not in ('balanced', 'balanced_sqrt'):
            return np.array([1.0, 1.0])
        n = len(y01)
        w = np.ones(2)
        for k in range(2):
            nk = int(np.sum(y01 == k))
            wk = n / (2 * max(nk, 1))
            if self.class_weight == 'balanced_sqrt':
                wk = wk ** 0.35
            w[k] = wk
        return w

    # ------------------------------------------------------------------
    # device plumbing
    # ------------------------------------------------------------------
    def _get_engine(self):
        idx = _device_index(self.device)
        if idx is None:
            idx = int(os.environ.get("LOCAL_RANK", 0)) if _dist() is not None else 0
        if self._engine is None or self._engine_dev != idx:
            self._engine = Engine(idx)
            self._engine_dev = idx
        return self._engine

    def _params_struct(self):
        policy = 0 if self.grow_policy == 'leaf' else 1
        self._mono_keep = None
        mono_ptr = None
        if self._mono_arr is not None:
            self._mono_keep = np.ascontiguousarray(self._mono_arr, dtype=np.int32)
            mono_ptr = self._mono_keep.ctypes.data
        prm = GbmParams(float(self.reg_lambda), float(self.gamma), float(self.min_child_weight),
                        float(self.learning_rate), int(self.min_samples_leaf), int(self.max_depth),
                        int(self.max_leaves), policy, mono_ptr)
        self._nan_keep = None
        if self.nan_direction == 'learn':
            prm, self._nan_keep = with_nan_direction(prm, self._nan_bin_id)
        return prm

    def _check_device_bins(self):
        mx = int(np.max(self.feature_bin_counts))
        if mx > 257:
            raise ValueError("the device path holds at most 257 bins per feature "
                             f"(feature with {mx} bins); use n_bins <= 256")

    def _tree_capacity(self):
        if self.grow_policy == 'leaf':
            return 2 * int(self.max_leaves) + 2
        return (1 << (int(self.max_depth) + 1)) - 1

    # ------------------------------------------------------------------
    # fit
    # ------------------------------------------------------------------
    def _check_supported(self):
        if self.objective not in ('auto', 'binary', 'regression'):
            raise NotImplementedError(f"objective={self.objective!r}: the B200 engine trains "
                                      "log-loss (binary, multi-class) and regression")
        if self.objective == 'regression' and self.loss not in ('mse', 'mae'):
            raise NotImplementedError(f"loss={self.loss!r}: regression takes 'mse' or 'mae'")
        if self.sampling_method != 'uniform':
            raise NotImplementedError("sampling_method='goss' is not on the B200 engine")
        if self.boosting_type != 'gbdt':
            raise NotImplementedError("boosting_type='dart' is not on the B200 engine")
        if self.custom_objective is not None:
            raise NotImplementedError("custom_objective is not on the B200 engine")
        if self.categorical_features is not None:
            raise NotImplementedError("categorical_features is not on the B200 engine")

    def fit(self, X, y, group=None, X_val=None, y_val=None, group_val=None, eval_set=None):
        try:
            import scipy.sparse
            if scipy.sparse.issparse(X):
                X = X.toarray()
            if X_val is not None and scipy.sparse.issparse(X_val):
                X_val = X_val.toarray()
        except ImportError:
            pass
        if self.max_depth != 'auto' and self.max_depth <= 0:
            raise ValueError(f"max_depth must be > 0, got {self.max_depth}")
        if self.learning_rate <= 0:
            raise ValueError(f"learning_rate must be > 0, got {self.learning_rate}")
        if self.n_estimators <= 0:
            raise ValueError(f"n_estimators must be > 0, got {self.n_estimators}")
        self._check_supported()
        if eval_set is not None and len(eval_set) > 0:
            X_val, y_val = eval_set[0]
        X = np.asarray(X)
        y = np.asarray(y)
        if X.ndim != 2:
            raise ValueError(f"X must be 2-D, got shape {X.shape}")
        if len(y) != X.shape[0]:
            raise ValueError(f"X has {X.shape[0]} rows but y has {len(y)}")
        if X.shape[0] == 0:
            raise ValueError("X is empty")
        regression = self.objective == 'regression'
        if regression:   # E:3113-3119
            self._is_multiclass = False
            self.classes_ = None
            self.n_classes_ = 1
            y = np.array(y, dtype=np.float64)
            if y_val is not None:
                y_val = np.array(y_val, dtype=np.float64)
        else:
            self.classes_ = np.unique(y)
            self.n_classes_ = len(self.classes_)
            if self.n_classes_ > 64:
                raise NotImplementedError("the B200 engine holds at most 64 classes")
            self._is_multiclass = self.n_classes_ > 2
            # class index of every label (classes_ is sorted and unique)
            y = np.searchsorted(self.classes_, y).astype(np.int64)
        if y_val is not None and not regression:
            y_val = np.asarray(y_val)
            yv = np.searchsorted(self.classes_, y_val)
            if np.any(yv >= len(self.classes_)) or np.any(self.classes_[np.minimum(yv, len(self.classes_) - 1)] != y_val):
                raise KeyError("y_val holds a label that is not in y")
            y_val = yv.astype(np.int64)
        if self.nan_direction not in ('left', 'learn'):
            raise ValueError(f"nan_direction must be 'left' or 'learn', got {self.nan_direction!r}")
        if self.nan_direction == 'learn' and (regression or self._is_multiclass):
            raise NotImplementedError("nan_direction='learn' is built for binary log-loss only")
        self.trees = []
        self._tree_nan_right = []
        self.mc_trees = None
        self.train_loss_history_ = []
        self.val_loss_history_ = []
        self.n_features_in_ = X.shape[1]
        if self.monotone_constraints is not None:
            mc = self.monotone_constraints
            if isinstance(mc, dict):
                arr = np.zeros(X.shape[1], dtype=np.int32)
                for f, d in mc.items():
                    arr[f] = d
                self._mono_arr = arr
            else:
                self._mono_arr = np.array(mc, dtype=np.int32)
            if len(self._mono_arr) != X.shape[1]:
                raise ValueError(f"monotone_constraints length ({len(self._mono_arr)}) must match "
                                 f"n_features ({X.shape[1]})")
        else:
            self._mono_arr = None
        self._categorical_set = set()
        self._is_categorical = np.zeros(X.shape[1], dtype=bool)
        if not np.issubdtype(X.dtype, np.floating) or X.dtype == np.float16:
            X = X.astype(np.float64)
        if X_val is not None:
            X_val = np.asarray(X_val)
            if not np.issubdtype(X_val.dtype, np.floating) or X_val.dtype == np.float16:
                X_val = X_val.astype(np.float64)
        self._compute_adaptive_hyperparameters(X, y)
        sample_weight = None
        if self.scale_pos_weight is not None and self.objective == 'binary':
            sample_weight = np.ones(len(y), dtype=np.float64)
            sample_weight[y == 1] = self.scale_pos_weight
        t0 = time.perf_counter()
        # Edges and bins are computed on the GPU (gbm_bin_edges /
        # gbm_upload_binned_rows) unless the edges are weighted
        # (scale_pos_weight), whose cumulative weights the host restatement
        # computes in NumPy's own summation order.
        on_device = sample_weight is None and 2 <= int(self.n_bins) <= 1023
        if on_device:
            eng = self._get_engine()
            self.bin_edges, self.feature_bin_counts, self._nan_bin_id = eng.bin_edges(X, self.n_bins)
        else:
            self.bin_edges, self.feature_bin_counts, self._nan_bin_id = binning.build_bin_edges(
                X, self.n_bins, None, sample_weight)
        self._max_bins = int(np.max(self.feature_bin_counts))
        self._check_device_bins()
        if on_device:
            lo, hi = _rank_rows(X.shape[0])
            _ensure_comm(eng)   # the upload all-reduces the bin occupancy (the skipped bin)
            eng.upload_binned_rows(lo, hi, self.bin_edges, self.feature_bin_counts, self._nan_bin_id)
            X_bin = _BinsOnDevice(X.shape)
        else:
            X_bin = binning.bin_features(X, self.bin_edges, self.feature_bin_counts, self._nan_bin_id)
        self.times['binning'] = (time.perf_counter() - t0) * 1000
        X_val_bin = None
        if X_val is not None and y_val is not None:
            if on_device:
                X_val_bin = eng.bin_features(X_val, self.bin_edges, self.feature_bin_counts,
                                             self._nan_bin_id)
            else:
                X_val_bin = binning.bin_features(X_val, self.bin_edges, self.feature_bin_counts,
                                                 self._nan_bin_id)
        t0 = time.perf_counter()
        if regression:
            self._fit_regression_device(X_bin, y, X_val_bin, y_val)
        elif self._is_multiclass:
            self._fit_multiclass_device(X_bin, y, X_val_bin, y_val)
        else:
            self._fit_binary_device(X_bin, y, X_val_bin, y_val)
        self.times['training'] = (time.perf_counter() - t0) * 1000
        self._pack_trees()
        self._compute_feature_importances()
        if self.verbose:
            print(f"\n  Training complete! ({self.n_trees_fitted_} trees)")
            print(f"    Binning:  {self.times['binning']:.2f} ms")
            print(f"    Training: {self.times['training']:.2f} ms")
        return self

    def fit_binned(self, X_bin, y01, counts, X_val_bin=None, y_val=None):
        """Train on a pre-binned matrix (bin ids per feature, ``counts`` bins each).

        The reference's own loop can be driven the same way
        (``_fit_binary`` on ``X_bin``, E:2825).  Hyper-parameters are used as
        given ('auto' values must already be resolved).
        """
        self._check_supported()
        y01 = np.asarray(y01).astype(np.int64)
        self.classes_ = np.array([0, 1])
        self.n_classes_ = 2
        self._is_multiclass = False
        self.n_features_in_ = X_bin.shape[1]
        self.feature_bin_counts = np.asarray(counts, dtype=np.int32)
        self._max_bins = int(np.max(self.feature_bin_counts))
        self._nan_bin_id = np.full(X_bin.shape[1], -1, dtype=np.int32)
        self._mono_arr = None
        self.trees = []
        self._tree_nan_right = []
        self.train_loss_history_ = []
        self.val_loss_history_ = []
        t0 = time.perf_counter()
        self._fit_binary_device(X_bin, y01, X_val_bin, y_val)
        self.times['training'] = (time.perf_counter() - t0) * 1000
        self._pack_trees()
        self._compute_feature_importances()
        return self

    def _fit_binary_device(self, X_bin, y, X_val_bin, y_val):
        """The reference's ``_fit_binary`` loop (E:2825-2944) with every round on the GPU."""
        n, p = X_bin.shape
        w2 = self._class_weight_pair(y)
        sw = w2[y]
        p0 = np.clip(np.average(y, weights=sw), 1e-7, 1.0 - 1e-7)
        self.base_score_ = float(np.log(p0 / (1.0 - p0)))
        n_sub = max(1, int(n * self.subsample))
        n_feat = max(1, int(p * self.colsample_bytree))
        seed = self.random_state
        if seed is None:
            seed = int.from_bytes(os.urandom(4), "little")
        if not (0 <= int(seed) <= 0xFFFFFFFF):
            raise ValueError("Seed must be between 0 and 2**32 - 1")
        sampler = Sampler(int(seed), n, p, n_sub, n_feat, self.subsample < 1.0,
                          self.colsample_bytree < 1.0, look_ahead=3)
        eng = self._get_engine()
        lo, hi = _rank_rows(n)
        _ensure_comm(eng)
        self._check_device_bins()
        t_up = time.perf_counter()
        if not isinstance(X_bin, _BinsOnDevice):
            # uint16 (the reference's bin dtype) and uint8 ids go up as they
            # are; the device clamps and narrows them
            Xr = X_bin[lo:hi]
            if Xr.dtype not in (np.uint8, np.uint16):
                Xr = binning.device_bins(Xr, self.feature_bin_counts)
            eng.upload_bins(Xr, self.feature_bin_counts)
        eng.upload_labels(y[lo:hi].astype(np.uint8), w2, self.base_score_, n_global=n)
        self.times['upload'] = (time.perf_counter() - t_up) * 1000
        self.scale_bits_ = eng.scale_bits()
        t_rounds = time.perf_counter()
        params = self._params_struct()
        cap = self._tree_capacity()
        F_val = np.full(len(y_val), self.base_score_) if y_val is not None else None
        best_val = np.inf
        no_improve = 0
        # Rounds are queued on the GPU in batches (gbm_fit_rounds); the
        # per-round bookkeeping below runs on each batch's results in order.
        # With early stopping a batch may train a few rounds past the stop;
        # they are dropped, so the kept trees are the reference's.
        batch = self.n_estimators if X_val_bin is None else 32
        try:
            m = 0
            stop = False
            while m < self.n_estimators and not stop:
                k = min(batch, self.n_estimators - m)
                for tree, loss in eng.fit_rounds(sampler, lo, params, cap, k):
                    self.trees.append(tree[:7])
                    self._tree_nan_right.append(tree[7][:tree[5]].copy() if len(tree) > 7 else None)
                    self.train_loss_history_.append(loss)
                    val_loss = None
                    if X_val_bin is not None:
                        F_val += self.learning_rate * _predict_tree_host(X_val_bin, tree)   # NaN direction included
                        val_loss = _logloss(y_val, F_val)
                        self.val_loss_history_.append(val_loss)
                    if self.verbose and ((m + 1) % 20 == 0 or m == 0):
                        msg = f"  Tree {m + 1:>3}/{self.n_estimators}  |  train-loss: {loss:.6f}"
                        if val_loss is not None:
                            msg += f"  |  val-loss: {val_loss:.6f}"
                        print(msg)
                    if self.early_stopping_rounds is not None and val_loss is not None:
                        if val_loss < best_val:
                            best_val = val_loss
                            self.best_iteration_ = m
                            no_improve = 0
                        else:
                            no_improve += 1
                            if no_improve >= self.early_stopping_rounds:
                                self.trees = self.trees[:self.best_iteration_ + 1]
                                self._tree_nan_right = self._tree_nan_right[:self.best_iteration_ + 1]
                                stop = True
                                break
                    m += 1
        finally:
            sampler.close()
        self.times['rounds'] = (time.perf_counter() - t_rounds) * 1000
        self.n_trees_fitted_ = len(self.trees)

    def _fit_regression_device(self, X_bin, y, X_val_bin, y_val):
        """The reference's ``_fit_regression`` loop (E:2607-2705) with every round
        on the GPU (gbm_round_reg_sampled): F from mean(y), g = F - y (mse) or
        sign(F - y) (mae), h = 1."""
        n, p = X_bin.shape
        self.init_score_ = float(np.mean(y))
        self.base_score_ = 0.0
        n_sub = max(1, int(n * self.subsample))
        n_feat = max(1, int(p * self.colsample_bytree))
        seed = self.random_state
        if seed is None:
            seed = int.from_bytes(os.urandom(4), "little")
        if not (0 <= int(seed) <= 0xFFFFFFFF):
            raise ValueError("Seed must be between 0 and 2**32 - 1")
        sampler = Sampler(int(seed), n, p, n_sub, n_feat, self.subsample < 1.0,
                          self.colsample_bytree < 1.0, look_ahead=3)
        eng = self._get_engine()
        lo, hi = _rank_rows(n)
        _ensure_comm(eng)
        self._check_device_bins()
        t_up = time.perf_counter()
        if not isinstance(X_bin, _BinsOnDevice):
            Xr = X_bin[lo:hi]
            if Xr.dtype not in (np.uint8, np.uint16):
                Xr = binning.device_bins(Xr, self.feature_bin_counts)
            eng.upload_bins(Xr, self.feature_bin_counts)
        eng.upload_targets(y[lo:hi], self.init_score_, self.loss, n_global=n)
        self.times['upload'] = (time.perf_counter() - t_up) * 1000
        params = self._params_struct()
        cap = self._tree_capacity()
        F_val = np.full(len(y_val), self.init_score_) if y_val is not None else None
        best_val, no_improve = np.inf, 0
        t_rounds = time.perf_counter()
        try:
            for m in range(self.n_estimators):
                # the round's shuffle applied on the device (the same sample as the host draw)
                tree, loss = eng.round_reg_sampled(sampler, lo, params, cap)
                self.trees.append(tree)
                self.train_loss_history_.append(loss)
                val_loss = None
                if F_val is not None:
                    F_val += self.learning_rate * _predict_tree_host(X_val_bin, tree)
                    val_loss = (np.mean((y_val - F_val) ** 2) if self.loss == 'mse'
                                else np.mean(np.abs(y_val - F_val)))
                    self.val_loss_history_.append(val_loss)
                if self.verbose and ((m + 1) % 20 == 0 or m == 0):
                    msg = f"  Tree {m + 1:>3}/{self.n_estimators}  |  train-loss: {loss:.6f}"
                    if val_loss is not None:
                        msg += f"  |  val-loss: {val_loss:.6f}"
                    print(msg)
                if self.early_stopping_rounds is not None and val_loss is not None:
                    if val_loss < best_val:
                        best_val, self.best_iteration_, no_improve = val_loss, m, 0
                    else:
                        no_improve += 1
                        if no_improve >= self.early_stopping_rounds:
                            self.trees = self.trees[:self.best_iteration_ + 1]
                            self._tree_nan_right = self._tree_nan_right[:self.best_iteration_ + 1]
                            break
        finally:
            sampler.close()
        self.times['rounds'] = (time.perf_counter() - t_rounds) * 1000
        self.n_trees_fitted_ = len(self.trees)

    def _class_weights_mc(self, y):
        """Per-class weights of ``_compute_class_weights`` (E:2570-2603) for K classes."""
        K = self.n_classes_
        n = len(y)
        w = np.ones(K, dtype=np.float64)
        if self.class_weight in ('balanced', 'balanced_sqrt'):
            for k in range(K):
                w_k = n / (K * max(int(np.sum(y == k)), 1))
                if self.class_weight == 'balanced_sqrt':
                    w_k = w_k ** 0.35
                w[k] = w_k
        return w

    def _fit_multiclass_device(self, X_bin, y, X_val_bin, y_val):
        """The reference's ``_fit_multiclass`` loop (E:2949-3065): per round one
        shared subsample and K trees, all on the GPU (gbm_round_mc_sampled)."""
        n, p = X_bin.shape
        K = self.n_classes_
        w = self._class_weights_mc(y)
        n_sub = max(1, int(n * self.subsample))
        n_feat = max(1, int(p * self.colsample_bytree))
        seed = self.random_state
        if seed is None:
            seed = int.from_bytes(os.urandom(4), "little")
        if not (0 <= int(seed) <= 0xFFFFFFFF):
            raise ValueError("Seed must be between 0 and 2**32 - 1")
        sampler = Sampler(int(seed), n, p, n_sub, n_feat, self.subsample < 1.0,
                          self.colsample_bytree < 1.0, look_ahead=3)
        eng = self._get_engine()
        lo, hi = _rank_rows(n)
        _ensure_comm(eng)
        self._check_device_bins()
        t_up = time.perf_counter()
        if not isinstance(X_bin, _BinsOnDevice):
            Xr = X_bin[lo:hi]
            if Xr.dtype not in (np.uint8, np.uint16):
                Xr = binning.device_bins(Xr, self.feature_bin_counts)
            eng.upload_bins(Xr, self.feature_bin_counts)
        eng.upload_labels_mc(y[lo:hi].astype(np.uint8), K, w, n_global=n)
        self.times['upload'] = (time.perf_counter() - t_up) * 1000
        self.scale_bits_ = eng.scale_bits()
        self.base_score_ = 0.0
        params = self._params_struct()
        cap = self._tree_capacity()
        self.mc_trees = [[] for _ in range(K)]
        F_val = np.zeros((len(y_val), K)) if y_val is not None else None
        yv_onehot = np.eye(K, dtype=np.float64)[y_val] if y_val is not None else None
        best_val, no_improve = np.inf, 0
        t_rounds = time.perf_counter()
        try:
            for m in range(self.n_estimators):
                # the round's shuffle applied on the device (the same sample as the host draw)
                trees, loss = eng.round_mc_sampled(sampler, lo, params, cap)
                for k in range(K):
                    self.mc_trees[k].append(trees[k])
                    if F_val is not None:
                        F_val[:, k] += self.learning_rate * _predict_tree_host(X_val_bin, trees[k])
                self.train_loss_history_.append(loss)
                val_loss = None
                if F_val is not None:
                    val_loss = _mc_logloss(yv_onehot, F_val)
                    self.val_loss_history_.append(val_loss)
                if self.verbose and ((m + 1) % 20 == 0 or m == 0):
                    msg = f"  Round {m + 1:>3}/{self.n_estimators}  |  {K} trees  |  train-loss: {loss:.6f}"
                    if val_loss is not None:
                        msg += f"  |  val-loss: {val_loss:.6f}"
                    print(msg)
                if self.early_stopping_rounds is not None and val_loss is not None:
                    if val_loss < best_val:
                        best_val, self.best_iteration_, no_improve = val_loss, m, 0
                    else:
                        no_improve += 1
                        if no_improve >= self.early_stopping_rounds:
                            for k in range(K):
                                self.mc_trees[k] = self.mc_trees[k][:self.best_iteration_ + 1]
                            break
        finally:
            sampler.close()
        self.times['rounds'] = (time.perf_counter() - t_rounds) * 1000
        self.trees = []
        self.n_trees_fitted_ = sum(len(t) for t in self.mc_trees)

    # ------------------------------------------------------------------
    # packing, importances (E:2192-2236, E:2343-2363)
    # ------------------------------------------------------------------
    def _pack_trees(self):
        if self._is_multiclass:
            self._mc_packed = [_pack_list(ts) for ts in self.mc_trees]
            return
        total = sum(t[5] for t in self.trees)
        feats = np.empty(total, dtype=np.int16)
        thr = np.empty(total, dtype=np.int64)
        vals = np.empty(total, dtype=np.float64)
        left = np.empty(total, dtype=np.int32)
        right = np.empty(total, dtype=np.int32)
        offs = np.empty(len(self.trees) + 1, dtype=np.int32)
        o = 0
        for t, (tf, tt, tv, tl, tr, nc, _) in enumerate(self.trees):
            offs[t] = o
            feats[o:o + nc] = tf[:nc]
            thr[o:o + nc] = tt[:nc]
            vals[o:o + nc] = tv[:nc]
            left[o:o + nc] = tl[:nc]
            right[o:o + nc] = tr[:nc]
            o += nc
        offs[len(self.trees)] = o
        self._packed_features, self._packed_thresholds = feats, thr
        self._packed_values, self._packed_left, self._packed_right = vals, left, right
        self._tree_offsets = offs
        self._packed_nan_right = None
        nrs = getattr(self, '_tree_nan_right', [])
        if any(x is not None for x in nrs):
            nr = np.zeros(total, dtype=np.uint8)
            for t, x in enumerate(nrs):
                if x is not None:
                    nr[offs[t]:offs[t] + len(x)] = x
            self._packed_nan_right = nr

    def _compute_feature_importances(self):
        gain = np.zeros(self.n_features_in_, dtype=np.float64)
        cnt = np.zeros(self.n_features_in_, dtype=np.int64)
        all_trees = [t for ts in self.mc_trees for t in ts] if self._is_multiclass else self.trees
        if all_trees:
            # every split's gain added to its feature in tree order, then node
            # order (np.add.at adds repeated indices one by one, in order: the
            # same float64 sums as the reference's loop)
            tf = np.concatenate([np.asarray(t[0])[:t[5]] for t in all_trees]).astype(np.int64)
            sg = np.concatenate([np.asarray(t[6], dtype=np.float64)[:t[5]] for t in all_trees])
            inner = tf >= 0
            np.add.at(gain, tf[inner], sg[inner])
            np.add.at(cnt, tf[inner], 1)
        tot = gain.sum()
        self.feature_importances_ = gain / tot if tot > 0 else np.zeros(self.n_features_in_)
        self.feature_split_counts_ = cnt

    # ------------------------------------------------------------------
    # predict (E:3274-3368)
    # ------------------------------------------------------------------
    def _packed(self):
        return {"features": self._packed_features, "thresholds": self._packed_thresholds,
                "values": self._packed_values, "left": self._packed_left,
                "right": self._packed_right, "offsets": self._tree_offsets,
                "nan_right": getattr(self, '_packed_nan_right', None)}

    def _prep_X(self, X):
        try:
            import scipy.sparse
            if scipy.sparse.issparse(X):
                X = X.toarray()
        except ImportError:
            pass
        if getattr(self, 'n_features_in_', None) is None:
            raise ValueError("This HybridHistGBMNumbaV1_0_1 instance is not fitted yet.")
        X = np.asarray(X)
        if not np.issubdtype(X.dtype, np.floating) or X.dtype == np.float16:
            X = X.astype(np.float64)
        if X.ndim != 2 or X.shape[1] != self.n_features_in_:
            raise ValueError(f"X has shape {X.shape}; the model has {self.n_features_in_} features")
        self._check_device_bins()
        return X

    def _proba_rows(self, X):
        """predict_proba of the rows of X on this rank's GPU: the rows are
        binned on the GPU (gbm_predict_raw) and go straight to the ensemble."""
        eng = self._get_engine()
        if self._is_multiclass:
            # K ensembles over the same binned rows, then the softmax (E:3290-3310, E:2328-2332)
            eng.predict_upload_raw(X, self.bin_edges, self.feature_bin_counts, self._nan_bin_id)
            F = np.zeros((X.shape[0], self.n_classes_))
            for k in range(self.n_classes_):
                eng.predict_set_model(self._mc_packed[k], len(self.mc_trees[k]), X.shape[1])
                eng.predict_run(self.learning_rate, 0.0)
                F[:, k] = eng.predict_fetch(want_F=True, want_proba=False)[0]
            return _softmax(F)
        _, proba = eng.predict_raw(X, self.bin_edges, self.feature_bin_counts, self._nan_bin_id,
                                   self._packed(), len(self.trees), self.learning_rate,
                                   getattr(self, 'base_score_', 0.0), want_F=False, want_proba=True)
        return np.column_stack([1 - proba, proba])

    def predict_proba(self, X):
        """predict_proba (E:3274-3336).  With torch.distributed running more
        than one rank, every rank passes the same X, predicts only its own
        contiguous block of rows on its own GPU (the ensemble is replicated;
        the walk needs no exchange), and the blocks are then all-gathered so
        every rank returns every row's probabilities.  predict_proba_local
        skips that gather."""
        X = self._prep_X(X)
        t0 = time.perf_counter()
        dist = _dist()
        if dist is None:
            out = self._proba_rows(X)
        else:
            lo, hi = _rank_rows(X.shape[0])
            out = _gather_rows(dist, self._proba_rows(X[lo:hi]), X.shape[0])
        self.times['inference'] = (time.perf_counter() - t0) * 1000
        return out

    def predict_proba_local(self, X):
        """This rank's block of rows of X (``_rank_rows``), predicted on this
        rank's GPU with no communication at all: ``(lo, hi, proba[hi - lo])``.
        The reference's parallel predict (predict_batch_parallel,
        E:3842-3883) splits rows over worker processes the same way; without
        torch.distributed the block is every row."""
        X = self._prep_X(X)
        lo, hi = _rank_rows(X.shape[0])
        return lo, hi, self._proba_rows(X[lo:hi])

    def predict_proba_binned(self, X_bin):
        """``predict_proba`` on bin ids already produced with this model's edges."""
        t0 = time.perf_counter()
        eng = self._get_engine()
        Xd = binning.device_bins(X_bin, self.feature_bin_counts)
        _, proba = eng.predict(Xd, self._packed(), len(self.trees), self.learning_rate,
                               getattr(self, 'base_score_', 0.0), want_F=False, want_proba=True)
        self.times['inference'] = (time.perf_counter() - t0) * 1000
        return np.column_stack([1 - proba, proba])

    def predict(self, X):
        if self.objective == 'regression':   # init score + the ensemble (E:3352-3360)
            X = self._prep_X(X)
            eng = self._get_engine()
            dist = _dist()
            lo, hi = _rank_rows(X.shape[0])   # row-sharded like predict_proba
            F, _ = eng.predict_raw(X[lo:hi], self.bin_edges, self.feature_bin_counts, self._nan_bin_id,
                                   self._packed(), len(self.trees), self.learning_rate,
                                   self.init_score_, want_F=True, want_proba=False)
            return F if dist is None else _gather_rows(dist, F[:, None], X.shape[0])[:, 0]
        proba = self.predict_proba(X)
        if self._is_multiclass:
            return self.classes_[np.argmax(proba, axis=1)]
        return self.classes_[(proba[:, 1] > 0.5).astype(int)]

    # ------------------------------------------------------------------
    # model JSON (E:4035-4205)
    # ------------------------------------------------------------------
    _RESOLVED = ('n_estimators', 'max_depth', 'learning_rate', 'n_bins', 'min_child_weight', 'gamma',
                 'subsample', 'colsample_bytree', 'max_leaves', 'reg_lambda', 'binning_strategy')

    def save_model(self, filepath):
        """JSON in the reference's layout (``save_model``, E:4035-4107), plus
        two keys the reference does not write: ``_nan_bin_id`` (the reference
        drops it and reloads every feature as NaN-free, E:4198-4200, which
        bins NaN rows differently after a reload) and ``resolved_params``
        (the hyper-parameters 'auto' resolved to, so a reloaded model predicts
        with the learning rate it was trained with).  The reference's
        ``load_model`` ignores both."""
        import json
        data = {
            'version': '1.2.2',
            'params': {},
            'n_classes_': int(self.n_classes_),
            'classes_': self.classes_.tolist() if self.classes_ is not None else None,
            'n_features_in_': int(self.n_features_in_) if self.n_features_in_ is not None else None,
            'objective': self.objective,
            '_is_multiclass': self._is_multiclass,
            'init_score_': float(self.init_score_),
            'base_score_': float(getattr(self, 'base_score_', 0.0)),
            'n_trees_fitted_': int(self.n_trees_fitted_),
            'best_iteration_': int(self.best_iteration_),
            'train_loss_history_': [float(x) for x in self.train_loss_history_],
            'val_loss_history_': [float(x) for x in self.val_loss_history_],
            '_max_bins': int(self._max_bins),
        }
        for k, v in self.get_params().items():
            if not callable(v):
                data['params'][k] = v
        if self.bin_edges is not None:
            data['bin_edges'] = np.asarray(self.bin_edges).tolist()
        if self.feature_bin_counts is not None:
            data['feature_bin_counts'] = np.asarray(self.feature_bin_counts).tolist()
        def tree_json(t):
            return {'features': np.asarray(t[0]).tolist(), 'thresholds': np.asarray(t[1]).tolist(),
                    'values': np.asarray(t[2]).tolist(), 'left': np.asarray(t[3]).tolist(),
                    'right': np.asarray(t[4]).tolist(), 'node_count': int(t[5]),
                    'split_gains': np.asarray(t[6]).tolist() if len(t) > 6 else []}
        if self._is_multiclass:
            data['mc_trees'] = [[tree_json(t) for t in ts] for ts in self.mc_trees]
        else:
            data['trees'] = [tree_json(t) for t in self.trees]
            nrs = getattr(self, '_tree_nan_right', [])
            if any(x is not None for x in nrs):   # nan_direction='learn' (no reference counterpart)
                data['nan_right'] = [[] if x is None else np.asarray(x).astype(int).tolist() for x in nrs]
        if self.feature_importances_ is not None:
            data['feature_importances_'] = np.asarray(self.feature_importances_).tolist()
        if self.feature_split_counts_ is not None:
            data['feature_split_counts_'] = np.asarray(self.feature_split_counts_).tolist()
        data['_categorical_set'] = list(self._categorical_set) if hasattr(self, '_categorical_set') else []
        if getattr(self, '_is_categorical', None) is not None:
            data['_is_categorical'] = np.asarray(self._is_categorical).tolist()
        if self._nan_bin_id is not None:
            data['_nan_bin_id'] = np.asarray(self._nan_bin_id).tolist()
        data['resolved_params'] = {k: getattr(self, k) for k in self._RESOLVED}
        with open(filepath, 'w') as f:
            json.dump(data, f)

    @classmethod
    def load_model(cls, filepath):
        """Loads a model written by :meth:`save_model` or by the reference's
        own ``save_model`` (``load_model``, E:4109-4205).  Without
        ``_nan_bin_id`` every feature is taken as NaN-free, as the reference
        does."""
        import json
        with open(filepath) as f:
            data = json.load(f)
        import inspect
        accepted = inspect.signature(cls.__init__).parameters   # a subclass may take fewer
        model = cls(**{k: v for k, v in data['params'].items() if k in accepted})
        model.n_classes_ = data['n_classes_']
        model.classes_ = np.array(data['classes_']) if data['classes_'] is not None else None
        model.n_features_in_ = data['n_features_in_']
        model.objective = data['objective']
        model._is_multiclass = data['_is_multiclass']
        model.init_score_ = data['init_score_']
        model.base_score_ = data.get('base_score_', 0.0)
        model.n_trees_fitted_ = data['n_trees_fitted_']
        model.best_iteration_ = data['best_iteration_']
        model.train_loss_history_ = data['train_loss_history_']
        model.val_loss_history_ = data['val_loss_history_']
        model._max_bins = data['_max_bins']
        if 'bin_edges' in data:
            model.bin_edges = np.array(data['bin_edges'], dtype=np.float64)
        if 'feature_bin_counts' in data:
            model.feature_bin_counts = np.array(data['feature_bin_counts'], dtype=np.int32)
        def tree_of(td):
            sg = np.array(td.get('split_gains', [0.0] * td['node_count']), dtype=np.float64)
            return (np.array(td['features'], dtype=np.int32), np.array(td['thresholds'], dtype=np.int64),
                    np.array(td['values'], dtype=np.float64), np.array(td['left'], dtype=np.int32),
                    np.array(td['right'], dtype=np.int32), int(td['node_count']), sg)
        model.trees = [tree_of(td) for td in data.get('trees', [])]
        nrs = data.get('nan_right')
        model._tree_nan_right = ([np.array(x, dtype=np.int32) if x else None for x in nrs] if nrs
                                 else [None] * len(model.trees))
        if 'mc_trees' in data:
            model.mc_trees = [[tree_of(td) for td in ts] for ts in data['mc_trees']]
        if 'feature_importances_' in data:
            model.feature_importances_ = np.array(data['feature_importances_'])
        if 'feature_split_counts_' in data:
            model.feature_split_counts_ = np.array(data['feature_split_counts_'])
        model._categorical_set = set(data.get('_categorical_set', []))
        if data.get('_is_categorical') is not None:
            model._is_categorical = np.array(data['_is_categorical'], dtype=np.bool_)
        model.binning_strategy = (model.binning_strategy_init if model.binning_strategy_init != 'auto'
                                  else 'standard')
        for k, v in data.get('resolved_params', {}).items():
            setattr(model, k, v)
        if data.get('_nan_bin_id') is not None:
            model._nan_bin_id = np.array(data['_nan_bin_id'], dtype=np.int32)
        elif model.n_features_in_ is not None:
            model._nan_bin_id = np.full(model.n_features_in_, -1, dtype=np.int32)
        model._pack_trees()
        return model

    def production_info(self):
        return {"engine": "libgbm_b200 (sm_100a)", "device": self.device,
                "n_trees": self.n_trees_fitted_, "n_features": self.n_features_in_}


def _softmax(F):
    """``_softmax`` (E:2328-2332)."""
    Fs = F - F.max(axis=1, keepdims=True)
    e = np.exp(Fs)
    return e / e.sum(axis=1, keepdims=True)


def _mc_logloss(y_onehot, F):
    """``_compute_multiclass_logloss`` (E:2335-2341)."""
    proba = np.clip(_softmax(F), 1e-15, 1 - 1e-15)
    return -np.mean(np.sum(y_onehot * np.log(proba), axis=1))


def _pack_list(trees):
    """``_pack_tree_list`` (E:2192-2216): one packed ensemble."""
    total = sum(t[5] for t in trees)
    out = {"features": np.empty(total, np.int16), "thresholds": np.empty(total, np.int64),
           "values": np.empty(total, np.float64), "left": np.empty(total, np.int32),
           "right": np.empty(total, np.int32), "offsets": np.empty(len(trees) + 1, np.int32)}
    o = 0
    for t, (tf, tt, tv, tl, tr, nc, _) in enumerate(trees):
        out["offsets"][t] = o
        out["features"][o:o + nc] = tf[:nc]
        out["thresholds"][o:o + nc] = tt[:nc]
        out["values"][o:o + nc] = tv[:nc]
        out["left"][o:o + nc] = tl[:nc]
        out["right"][o:o + nc] = tr[:nc]
        o += nc
    out["offsets"][len(trees)] = o
    return out


class _BinsOnDevice:
    """Stands for a training matrix that was binned straight into the engine."""

    def __init__(self, shape):
        self.shape = shape


def _ensure_comm(eng):
    """One NCCL communicator per engine across fits, made when torch.distributed
    runs more than one rank (before any upload: the bin upload all-reduces)."""
    dist = _dist()
    if dist is None:
        return
    ws, rk = dist.get_world_size(), dist.get_rank()
    if getattr(eng, "_comm_world", None) != (ws, rk):
        uid = [Engine.nccl_unique_id() if rk == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eng.init_comm(uid[0], ws, rk)


def _rank_rows(n):
    """This rank's contiguous block of rows (all rows without torch.distributed)."""
    dist = _dist()
    if dist is None:
        return 0, n
    ws, rk = dist.get_world_size(), dist.get_rank()
    return (n * rk) // ws, (n * (rk + 1)) // ws


def _gather_rows(dist, local, n):
    """Every rank's block of rows (``_rank_rows`` order) of a float64 [m, k]
    array, all-gathered so each rank holds all n rows.  Only the results
    travel: blocks are padded to the largest block and exchanged as one
    tensor (on this rank's GPU under NCCL, on the host under gloo)."""
    import torch
    ws = dist.get_world_size()
    k = local.shape[1]
    bounds = [((n * r) // ws, (n * (r + 1)) // ws) for r in range(ws)]
    m = max(h - l for l, h in bounds)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    buf = torch.zeros((m, k), dtype=torch.float64, device=dev)
    buf[:local.shape[0]] = torch.from_numpy(np.ascontiguousarray(local)).to(dev)
    allb = torch.empty((ws * m, k), dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(allb, buf)
    allb = allb.cpu().numpy()
    return np.concatenate([allb[r * m:r * m + (h - l)] for r, (l, h) in enumerate(bounds)], axis=0)


def _predict_tree_host(X_bin, tree):
    """Values of one tree for every row (host, used for the small validation set);
    a tree with an 8th element sends the NaN bin right where it is 1."""
    tf, tt, tv, tl, tr, nc, _ = tree[:7]
    nr = np.asarray(tree[7]) if len(tree) > 7 else np.zeros(len(tf), np.int32)
    node = np.zeros(X_bin.shape[0], dtype=np.int64)
    rows = np.arange(X_bin.shape[0])
    while True:
        f = tf[node]
        act = f >= 0
        if not act.any():
            break
        ff = np.where(act, f, 0)
        b = X_bin[rows, ff].astype(np.int64)
        go_left = (b <= tt[node]) & ~((nr[node] != 0) & (b == 0))
        node = np.where(act, np.where(go_left, tl[node], tr[node]), node)
    return tv[node]


def _logloss(y, F):
    p = 1.0 / (1.0 + np.exp(-np.clip(F, -500, 500)))
    p = np.clip(p, 1e-15, 1 - 1e-15)
    return -np.mean(y * np.log(p) + (1 - y) * np.log(1 - p))


class HybridHistGBMRegressorV1_0_1(HybridHistGBMNumbaV1_0_1):
    """The reference's regressor (objective='regression', mse or mae) on the B200 engine."""

    def __init__(self, n_estimators='auto', max_depth='auto', learning_rate='auto',
                 n_bins='auto', reg_lambda=1.0, min_samples_leaf=5,
                 min_child_weight='auto', gamma='auto',
                 subsample='auto', colsample_bytree='auto',
                 grow_policy='leaf', max_leaves=31, binning_strategy='auto',
                 monotone_constraints=None, categorical_features=None,
                 early_stopping_rounds=None, verbose=True, random_state=None,
                 loss='mse', device='b200'):
        super().__init__(
            n_estimators=n_estimators, max_depth=max_depth, learning_rate=learning_rate,
            n_bins=n_bins, reg_lambda=reg_lambda, min_samples_leaf=min_samples_leaf,
            min_child_weight=min_child_weight, gamma=gamma, subsample=subsample,
            colsample_bytree=colsample_bytree, class_weight=None, grow_policy=grow_policy,
            max_leaves=max_leaves, binning_strategy=binning_strategy,
            monotone_constraints=monotone_constraints, categorical_features=categorical_features,
            early_stopping_rounds=early_stopping_rounds, verbose=verbose, random_state=random_state,
            objective='regression', focal_gamma=2.0, loss=loss, device=device)
