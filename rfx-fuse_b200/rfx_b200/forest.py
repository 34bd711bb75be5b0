"""Drop-in estimators with the RFXFuse Python surface (python/randomforest_py.cpp).

RandomForestClassifier / RandomForestRegressor / RandomForestUnsupervised keep the
reference constructor arguments and defaults, and resolve them the same way
(python/randomforest_py.cpp:1270-1320, 1367-1500, 3066-3240, 4628-5040).  ``fit`` runs the
whole forest on the GPU through librfx_b200.so; the getters return what the reference's
getters return.  ``show_progress`` draws the reference's tqdm bar (one update per batch of
trees).  Arguments that only select among the reference's own implementations (use_gpu,
use_sparse, gpu_loss_function, ...) are accepted and ignored: there is one implementation
here, the device one.
"""
from __future__ import annotations

import enum
import math

import numpy as np

from . import _abi as A


class TaskType(enum.IntEnum):
    """The reference's task enum (include/rf_random_forest.hpp:29-33)."""
    CLASSIFICATION = A.TASK_CLASSIFICATION
    REGRESSION = A.TASK_REGRESSION
    UNSUPERVISED = A.TASK_UNSUPERVISED

MAX_NODE_CAP = 32001


def calculate_maxnode(nsample: int, minndsize: int, user_maxnode: int = 0) -> int:
    """include/rf_config.hpp:15-32."""
    if user_maxnode > 0:
        return int(user_maxnode)
    m = max(int(minndsize), 1)
    leaves = (int(nsample) + m - 1) // m
    return min(2 * leaves + 1, MAX_NODE_CAP)


def _isqrt_f32(x: int) -> int:
    # static_cast<integer_t>(std::sqrt(static_cast<real_t>(x)))
    return int(np.sqrt(np.float32(x), dtype=np.float32))


def feature_kinds(task: int, X: np.ndarray, maxcat: int, categorical_features=None) -> np.ndarray:
    """cat[] of a fit: only the classifier's fit detects categorical columns
    (python/randomforest_py.cpp:1415-1499); the regressor and the unsupervised forest never
    call set_categorical_features, so every feature stays quantitative (cat = 1,
    src/rf_random_forest.cpp:461)."""
    if task != A.TASK_CLASSIFICATION:
        return np.ones(X.shape[1], np.int32)
    return detect_categorical(X, maxcat, categorical_features)


def detect_categorical(X: np.ndarray, maxcat: int, categorical_features=None) -> np.ndarray:
    """cat[] exactly as RandomForestClassifier::fit builds it (python/randomforest_py.cpp:1413-1460)."""
    n, p = X.shape
    cat = np.ones(p, np.int32)
    if categorical_features is not None:
        for c in list(categorical_features):
            c = int(c)
            if 0 <= c < p:
                cat[c] = len(np.unique(X[:, c]))
        return cat
    for m in range(p):
        col = X[:, m]
        u = np.unique(col)
        all_int = not np.any(np.abs(col - np.round(col)) > np.float32(1e-5))
        mn = min(np.float32(1e10), col.min()) if n else np.float32(1e10)
        mx = max(np.float32(-1e10), col.max()) if n else np.float32(-1e10)
        if all_int and 2 < len(u) <= maxcat and mn >= 0.0 and mx < np.float32(maxcat):
            cat[m] = len(u)
    return cat


class _Forest:
    _task = None

    def __init__(self, nsample=1000, ntree=100, mdim=10, nclass=2, maxcat=10, mtry=0,
                 maxnode=0, minndsize=1, ncsplit=25, ncmax=25, iseed=12345,
                 compute_proximity=False, compute_importance=True,
                 compute_local_importance=False, use_gpu=False, use_qlora=False,
                 quant_mode="nf4", use_sparse=False, sparsity_threshold=1e-6, batch_size=0,
                 nodesize=5, cutoff=0.01, show_progress=True, progress_desc="",
                 gpu_loss_function="gini", rank=32, power_iterations=30, n_threads_cpu=0,
                 use_rfgap=False, importance_method="local_imp", clique_M=-1,
                 use_casewise=False, compute_proximity_importance=False,
                 compute_leaf_assignments=False, categorical_features=None,
                 use_histogram=True, n_bins=256, class_weight="", classwt=None,
                 device=0, prox_rows=0, batch_trees=0, lowrank_oversample=16,
                 lowrank_power_iters=1, synthetic_ratio=1.0):
        if use_casewise:
            raise NotImplementedError("use_casewise=True is not implemented on the device path")
        if use_rfgap:
            raise NotImplementedError("RF-GAP proximity is not implemented on the device path")
        if compute_local_importance:
            raise NotImplementedError("local importance is not implemented on the device path")
        if not use_histogram:
            raise NotImplementedError("only the histogram grower exists on the device path")
        self.nsample = int(nsample)
        self.ntree = int(ntree)
        self.mdim = int(mdim)
        self.maxcat = int(maxcat)
        self.minndsize = int(minndsize)
        self.iseed = int(iseed)
        self.compute_proximity = bool(compute_proximity)
        self.compute_importance = bool(compute_importance)
        self.use_qlora = bool(use_qlora)
        self.quant_mode = str(quant_mode)
        self.rank = int(rank)
        self.lowrank_oversample = int(lowrank_oversample)
        self.lowrank_power_iters = int(lowrank_power_iters)
        if self.use_qlora and self.compute_proximity:
            if self.quant_mode.lower() != "int8":
                raise NotImplementedError("low-rank proximity is stored as int8 factors: "
                                          "use quant_mode='int8'")
            if not 1 <= self.rank <= 64:
                raise NotImplementedError("low-rank proximity rank must be in [1, 64]")
        self.n_bins = min(int(n_bins), 256)
        self.categorical_features = categorical_features
        self.class_weight = class_weight
        self.classwt = classwt
        self.device = int(device)
        self.prox_rows = int(prox_rows)
        self.batch_trees = int(batch_trees)
        self.nodesize = int(nodesize)  # stored, never read by the growers (as in the reference)
        self.show_progress, self.progress_desc = bool(show_progress), str(progress_desc)
        # stored as given, for the model file (model_io): not used by the device path
        self.ncsplit, self.ncmax = int(ncsplit), int(ncmax)
        self.use_gpu, self.use_sparse = bool(use_gpu), bool(use_sparse)
        self.sparsity_threshold, self.cutoff = float(sparsity_threshold), float(cutoff)
        self.batch_size, self.n_threads_cpu = int(batch_size), int(n_threads_cpu)
        self.gpu_loss_function, self.power_iterations = str(gpu_loss_function), int(power_iterations)
        self.importance_method, self.clique_M = str(importance_method), int(clique_M)
        self.compute_proximity_importance = bool(compute_proximity_importance)
        self.compute_leaf_assignments = bool(compute_leaf_assignments)
        self.synthetic_ratio = float(synthetic_ratio)
        self._mtry_arg = int(mtry)
        self._maxnode = calculate_maxnode(self.nsample, self.minndsize, int(maxnode))
        self._mtry = self._resolve_mtry_ctor(int(mtry))
        self._ctx = None
        self._fitted = False

    def _progress_bar(self, total):
        """The reference wrapper's tqdm bar (python/randomforest_py.cpp:1560-1600), or None."""
        if not self.show_progress:
            return None
        try:
            import tqdm
        except ImportError:
            return None
        return tqdm.tqdm(total=total, desc=self.progress_desc, unit="tree", unit_scale=False,
                         leave=False, dynamic_ncols=True, miniters=1,
                         bar_format="{desc}: {percentage:3.0f}%|{bar}| {n}/{total} {unit} "
                                    "[{elapsed}<{remaining}, {rate_fmt}]")

    # ---- resolution rules of the reference wrappers
    def _resolve_mtry_ctor(self, mtry):
        return mtry if mtry > 0 else _isqrt_f32(self.mdim)

    def _lowrank_rank(self):
        return self.rank if (self.use_qlora and self.compute_proximity) else 0

    def _context(self):
        if self._ctx is None:
            self._ctx = A.Context(self.device)
        return self._ctx

    def _fit(self, X, y, sample_weights, task, mtry, maxnode, classwt):
        X = np.ascontiguousarray(X, dtype=np.float32)
        if X.ndim != 2:
            raise RuntimeError("X must be 2-dimensional (samples, features)")
        n, p = X.shape
        self.n_features_ = p
        cat = feature_kinds(task, X, self.maxcat, self.categorical_features)
        self._cat = cat
        prm = A.FitParams(task, n, p, mtry, self.minndsize, maxnode, self.iseed, 12345,
                          self.n_bins, self.maxcat, int(self.compute_importance),
                          int(self.compute_proximity), self.prox_rows, self.batch_trees, 0,
                          self._lowrank_rank(),
                          int(task != A.TASK_UNSUPERVISED or self.compute_leaf_assignments),
                          int(self.compute_leaf_assignments), 1)
        ycls = yreg = sw = cw = None
        if task == A.TASK_CLASSIFICATION:
            ycls = np.ascontiguousarray(y, dtype=np.int32)
        elif task == A.TASK_REGRESSION:
            yreg = np.ascontiguousarray(y, dtype=np.float32)
        if sample_weights is not None and len(sample_weights) > 0:
            sw = np.ascontiguousarray(sample_weights, dtype=np.float32)
        if classwt is not None:
            cw = np.ascontiguousarray(classwt, dtype=np.float32)
        inp = A.Inputs(A.ptr(X, A._pf), A.ptr(ycls, A._pi), A.ptr(yreg, A._pf), A.ptr(sw, A._pf),
                       A.ptr(cat, A._pi), A.ptr(cw, A._pf))
        N = 2 * n if task == A.TASK_UNSUPERVISED else n
        T, M = self.ntree, maxnode
        # the tree arrays stay in the device tree store (keep_trees); trees_ fetches them on
        # first use.  Only the node counts and the per-tree importance rows come back now.
        tr = {"nnode": np.zeros(T, np.int32), "tree_rr": np.zeros((T, p), np.float32),
              "tree_used": np.zeros((T, p), np.uint8)}
        trees = A.Trees(None, None, None, None, None, A.ptr(tr["nnode"], A._pi), None, None,
                        None, None, A.ptr(tr["tree_rr"], A._pf), A.ptr(tr["tree_used"], A._pu8))
        ctx = self._context()
        ctx.load(prm, inp)
        bar = self._progress_bar(T)
        try:
            if bar is not None:
                def _update(done, _total):
                    bar.update(done - bar.n)
                    return False
                ctx.set_progress(_update)
            ctx.grow(0, T, trees)
        finally:
            if bar is not None:
                ctx.set_progress(None)
                bar.close()
        ncl = {A.TASK_REGRESSION: 1, A.TASK_UNSUPERVISED: 2}.get(task)
        if ncl is None:
            ncl = len(np.unique(ycls))
        acc = {"nout": np.zeros(N, np.int32), "votes": np.zeros((N, ncl), np.int32),
               "q": np.zeros((N, ncl), np.float32), "oob_sum": np.zeros(N, np.float32),
               "avimp": np.zeros(p, np.float32), "sqsd": np.zeros(p, np.float32),
               "labels": np.zeros(N, np.int32)}
        ac = A.Accum(0, 0, *[A.ptr(acc[k], t) for k, t in (
            ("nout", A._pi), ("votes", A._pi), ("q", A._pf), ("oob_sum", A._pf), ("avimp", A._pf),
            ("sqsd", A._pf), ("labels", A._pi))])
        if ncl == 1:
            ac.votes = None
            ac.q = None
            ac.labels = None
        ctx.results(ac)
        if self._lowrank_rank():
            ctx.lowrank_build(self.rank, self.lowrank_oversample, self.lowrank_power_iters,
                              seed=self.iseed)
        self._trees = tr
        self._trees_full = False
        self.acc_ = acc
        self.n_rows_ = N
        self.nclass_ = ncl
        self._task_id = task
        self._maxnode_eff = M
        self._mtry_eff = mtry
        self._fitted = True
        self._finalize(y)
        return None

    @property
    def trees_(self):
        """The forest's tree arrays in the reference layout ([ntree, maxnode]; treemap
        [ntree, 2 maxnode]), copied from the device tree store on first use."""
        if not getattr(self, "_trees_full", True):
            T, M = self.ntree, self._maxnode_eff
            tr = self._trees
            for k, shape, dt in (("nodestatus", (T, M), np.int32), ("bestvar", (T, M), np.int32),
                                 ("xbestsplit", (T, M), np.float32),
                                 ("treemap", (T, 2 * M), np.int32),
                                 ("nodeclass", (T, M), np.int32),
                                 ("nodepred", (T, M), np.float32),
                                 ("tnodewt", (T, M), np.float32)):
                tr[k] = np.empty(shape, dt)
            self._context().get_trees(0, T, A.Trees(*[A.ptr(tr[k], t) for k, t in (
                ("nodestatus", A._pi), ("bestvar", A._pi), ("xbestsplit", A._pf),
                ("treemap", A._pi), ("nodeclass", A._pi), ("nnode", A._pi),
                ("nodepred", A._pf), ("tnodewt", A._pf))], None, None, None, None))
            self._trees_full = True
        return self._trees

    @trees_.setter
    def trees_(self, value):
        self._trees = value
        self._trees_full = True

    def _finalize(self, y):
        acc = self.acc_
        nout = acc["nout"]
        # feature importance: finalize_training (src/rf_random_forest.cpp:2690-2698)
        av = acc["avimp"]
        s = np.add.accumulate(np.abs(av), dtype=np.float32)[-1] if len(av) else np.float32(0)
        self._importances = av.copy() if s > 0 else np.zeros_like(av)

    def _check(self):
        if not self._fitted:
            raise RuntimeError("Model must be fitted first")

    def save(self, filepath):
        """Write the model as the reference's RFX0 v1 file (RandomForest::save,
        src/rf_random_forest.cpp:6037-6140); RFXFuse.load() reads it."""
        if not self._fitted:
            raise RuntimeError("Model must be fitted before saving")
        from . import model_io
        model_io.write(str(filepath), model_io.from_estimator(self))

    # ---- reference getters
    def feature_importances_(self):
        self._check()
        return self._importances.copy()

    def get_oob_error(self):
        self._check()
        return float(self._oob_error)

    def get_oob_counts(self):
        self._check()
        return self.acc_["nout"].copy()

    def get_n_samples(self):
        return self.n_rows_

    def get_n_features(self):
        return self.n_features_

    def get_n_classes(self):
        return self.nclass_

    def get_task_type(self):
        return TaskType(self._TASK)

    def cleanup(self):
        """The reference frees its process-wide GPU pools here; this library keeps no memory
        outside the model's own context, so there is nothing to release."""
        return None

    def compute_proximity_matrix(self):
        """Alias of get_proximity_matrix (python/randomforest_py.cpp:2880)."""
        return self.get_proximity_matrix()

    def get_proximity_matrix(self):
        """Dense float32 finishprox'd proximity (python/randomforest_py.cpp:2129-2181)."""
        self._check()
        if not self.compute_proximity:
            raise RuntimeError("Proximity was not computed (compute_proximity=False)")
        if self._lowrank_rank():
            raise RuntimeError(
                "Proximity matrix not available in full form. Low-rank mode is active "
                "(use_qlora=True). Proximity is stored in low-rank factors (A and B). Use "
                "get_lowrank_factors() instead, or disable use_qlora for datasets whose full "
                "matrix fits.")
        ctx = self._context()
        _, length = ctx.prox_buffer()
        R = int(round((1 + math.sqrt(1 + 8 * length)) / 2)) if length else (
            self.prox_rows or self.n_rows_)
        if getattr(self, "_sharded_prox", None) is not None:
            # reduce-scattered counts of a tree-sharded fit: a collective over its ranks
            from .shard import sharded_proximity_dense
            return sharded_proximity_dense(self)
        out = np.empty((R, R), np.float32)
        ctx.prox_dense(0, R, out)
        return out

    # ---- low-rank proximity (use_qlora=True, quant_mode="int8")
    def _check_lowrank(self):
        self._check()
        if not self._lowrank_rank():
            raise RuntimeError(
                "Low-rank factors not available. Either low-rank mode is not active "
                "(use_qlora=True required), or factors have not been computed yet.")

    def get_lowrank_factors(self):
        """(A float64 [n, r], B float64 [n, r], r) with proximity ~ A B^T and B = A, the
        dequantised int8 factors (python/randomforest_py.cpp:2183-2223)."""
        self._check_lowrank()
        Af, _, _ = self._context().lowrank_factors()
        A64 = Af.astype(np.float64)
        return A64, A64.copy(), int(Af.shape[1])

    def get_lowrank_quantized(self):
        """(q int8 [n, r], scale float32 [n]): A_i = scale_i * q_i."""
        self._check_lowrank()
        _, q, s = self._context().lowrank_factors()
        return q, s

    def get_lowrank_topk(self, k=50, row_begin=0, row_end=None):
        """Top-k neighbours of every row under the quantised low-rank proximity, j != i:
        (indices int32 [rows, k], values float32 [rows, k]), value descending."""
        self._check_lowrank()
        R = self._lowrank_rows()
        dist = getattr(self, "_shard_dist", None)
        if dist is not None and row_begin == 0 and row_end is None:
            from .shard import lowrank_topk_sharded  # collective over the fit's ranks
            return lowrank_topk_sharded(self, k, dist)
        row_end = R if row_end is None else int(row_end)
        return self._context().lowrank_topk(int(k), int(row_begin), row_end)

    def get_lowrank_product(self, row_begin=0, row_end=None):
        """Rows of the reconstructed low-rank proximity (scale_i scale_j q_i . q_j)."""
        self._check_lowrank()
        R = self._lowrank_rows()
        row_end = R if row_end is None else int(row_end)
        return self._context().lowrank_product(int(row_begin), row_end, R)

    def _lowrank_rows(self):
        return self.prox_rows if self.prox_rows else self.n_rows_

    def get_proximity_counts(self):
        """Packed upper triangle (i < j) of the integer OOB x in-bag co-membership counts."""
        self._check()
        ctx = self._context()
        dev, length = ctx.prox_buffer()
        out = np.empty(length, np.int32)
        if length:
            ctx.copy_to_host(out, dev)
        return out

    # ---- leaf assignments, similar rows, outliers (include/rf_random_forest.hpp:296-365) ----
    _NO_LEAVES = ("Leaf assignments not available. Set compute_leaf_assignments=True when "
                  "creating the model.")

    def _check_leaves(self):
        self._check()
        if not self.compute_leaf_assignments:
            raise RuntimeError(self._NO_LEAVES)

    def get_leaf_assignments(self):
        """int16 [ntree, n_samples]: terminal node of every training row in every tree."""
        self._check_leaves()
        return self._context().leaf_assignments()

    def build_inverted_leaf_index(self):
        self._check_leaves()
        self._context().leaf_index()
        self._leaf_index_built = True

    def has_inverted_leaf_index(self):
        return bool(getattr(self, "_leaf_index_built", False))

    def get_top_k_similar(self, query_idx, k=10, exclude_self=True):
        """(indices int32, similarities float32) of the training rows sharing the query's
        leaf most often over the trees where the query was OOB."""
        self._check_leaves()
        self._leaf_index_built = True  # built on first use, as the reference's binding does
        (idx, sim), = self._context().leaf_top_k_similar([int(query_idx)], int(k), exclude_self)
        if idx.shape[0] == 0:
            raise RuntimeError(self._NO_LEAVES)
        return idx, sim

    def compute_proximity_from_leaves(self, sample_i, sample_j):
        self._check_leaves()
        return self._context().leaf_proximity(int(sample_i), int(sample_j))

    def predict_leaf_assignments(self, X):
        """int16 [n_new, ntree] terminal nodes of new rows."""
        self._check()
        X = np.ascontiguousarray(X, dtype=np.float32)
        if X.ndim != 2:
            raise RuntimeError("X must be 2-dimensional")
        return self._context().predict_leaves(X, self.ntree)

    def predict_top_k_similar(self, X, k=10):
        """(indices int32 [n_new, k], similarities float32 [n_new, k]) over all trees."""
        self._check_leaves()
        self._leaf_index_built = True
        X = np.ascontiguousarray(X, dtype=np.float32)
        if X.ndim != 2:
            raise RuntimeError("X must be 2-dimensional")
        return self._context().predict_top_k_similar(X, int(k))

    def select_outlier_anchors(self, n_anchors=100, method="random"):
        self._check_leaves()
        a = self._context().select_anchors(int(n_anchors), 1 if method == "diverse" else 0,
                                           self.iseed)
        self._outlier_anchors = a
        return a.copy()

    def compute_outlier_scores(self, mode="full", n_anchors=100):
        """Breiman-Cutler outlier scores ((raw - median) / MAD; per class for a classifier)."""
        self._check_leaves()
        anchors = None
        if mode == "greedy":
            a = getattr(self, "_outlier_anchors", None)
            if a is None or len(a) == 0 or len(a) != int(n_anchors):
                self.select_outlier_anchors(int(n_anchors), "random")
            anchors = self._outlier_anchors
        labels = self.acc_["labels"] if self._task_id == A.TASK_CLASSIFICATION else None
        self._leaf_index_built = True
        scores, _raw = self._context().outlier_scores(1 if mode == "greedy" else 0, anchors,
                                                      int(n_anchors), labels, self.n_rows_)
        self.outlier_scores_ = scores
        return scores

    def predict_outlier_scores(self, X, mode="full", n_anchors=100):
        """Outlier scores of new rows against the training rows, normalised with the
        statistics of the last compute_outlier_scores (per predicted class for a classifier)."""
        self._check_leaves()
        if getattr(self, "outlier_scores_", None) is None:
            raise RuntimeError("Outlier normalization stats not available. Call "
                               "compute_outlier_scores() on training data first.")
        X = np.ascontiguousarray(X, dtype=np.float32)
        if X.ndim != 2:
            raise RuntimeError("X must be 2-dimensional")
        classes = None
        if self._task_id == A.TASK_CLASSIFICATION:
            classes = np.searchsorted(self.classes_, self.predict(X)).astype(np.int32)
        self._leaf_index_built = True
        return self._context().predict_outlier_scores(X, 1 if mode == "greedy" else 0,
                                                      int(n_anchors), classes)

    def compute_outliers(self, k=10, mode="full", n_anchors=100):
        """(indices, scores) of the k highest outlier scores."""
        scores = self.compute_outlier_scores(mode, n_anchors)
        return A.rank_scores_desc(scores, int(k))


def _argmax_last(q: np.ndarray) -> np.ndarray:
    """argmax with the reference's `>=` scan: ties go to the highest class index."""
    k = q.shape[1]
    return (k - 1 - np.argmax(q[:, ::-1], axis=1)).astype(np.int32)


class _Classifying(_Forest):
    def _class_error_and_preds(self, labels0):
        acc = self.acc_
        q = acc["q"]
        nout = acc["nout"]
        oob = nout > 0
        pred = _argmax_last(q)
        # compute_classification_error (src/rf_random_forest.cpp:3947-4012)
        tot = int(oob.sum())
        correct = int((pred[oob] == labels0[oob]).sum())
        self._oob_error = (np.float32(1.0) - np.float32(correct) / np.float32(tot)) if tot else np.float32(0)
        # compute_oob_predictions (src/rf_random_forest.cpp:3776-3840)
        self._oob_class = np.where(oob, pred, 0).astype(np.int32)
        tv = np.add.accumulate(q, axis=1, dtype=np.float32)[:, -1] if q.shape[1] else np.zeros(len(q), np.float32)
        probs = np.full(q.shape, np.float32(1.0) / np.float32(q.shape[1]), np.float32)
        ok = oob & (tv > 0)
        probs[ok] = q[ok] / tv[ok, None]
        self._oob_proba = probs

    def get_oob_predictions(self):
        self._check()
        return self._oob_class.astype(np.float32)


class RandomForestClassifier(_Classifying):
    _TASK = A.TASK_CLASSIFICATION
    _task = A.TASK_CLASSIFICATION

    def _is_training_size(self, X):
        # predict_classification / predict_proba treat any input with nsample rows as the
        # training data and return the stored OOB results (src/rf_random_forest.cpp:3384-3401)
        return np.asarray(X).shape[0] == self.nsample

    def predict(self, X):
        """Class labels (python/randomforest_py.cpp:1860-1869)."""
        self._check()
        if self._is_training_size(X):
            return self.classes_[self._oob_class].astype(np.int32)
        cls, _ = self._context().predict(np.ascontiguousarray(X, np.float32), self.nclass_)
        return self.classes_[cls].astype(np.int32)

    def predict_proba(self, X):
        """Class probabilities [n, nclass] (python/randomforest_py.cpp:1871-1880)."""
        self._check()
        if self._is_training_size(X):
            return self._oob_proba.copy()
        _, proba = self._context().predict(np.ascontiguousarray(X, np.float32), self.nclass_)
        return proba

    def fit(self, X, y, sample_weights=None):
        y = np.ascontiguousarray(y, dtype=np.int32)
        ncl = len(np.unique(y))
        classwt = None
        if self.classwt is not None:
            classwt = np.ascontiguousarray(self.classwt, dtype=np.float32)
            if classwt.shape[0] != ncl:
                raise RuntimeError(f"classwt length ({classwt.shape[0]}) must match number of classes ({ncl})")
        elif self.class_weight == "balanced":
            counts = np.zeros(ncl, np.int64)
            for c in y:
                if 0 <= c < ncl:
                    counts[c] += 1
            n = np.float32(len(y))
            classwt = np.array([n / (np.float32(ncl) * np.float32(k)) if k > 0 else np.float32(1.0)
                                for k in counts], np.float32)
        self.classwt_ = classwt
        self.classes_ = np.unique(y).astype(np.int32)
        self._fit(X, y, sample_weights, A.TASK_CLASSIFICATION, self._mtry, self._maxnode, classwt)

    def _finalize(self, y):
        super()._finalize(y)
        self._class_error_and_preds(self.acc_["labels"])


class RandomForestRegressor(_Forest):
    _TASK = A.TASK_REGRESSION
    _task = A.TASK_REGRESSION

    def __init__(self, *args, **kw):
        kw.setdefault("compute_proximity", False)
        kw.setdefault("gpu_loss_function", "mse")
        super().__init__(*args, **kw)

    def fit(self, X, y, sample_weights=None):
        self._y = np.ascontiguousarray(y, dtype=np.float32)
        self._fit(X, self._y, sample_weights, A.TASK_REGRESSION, self._mtry, self._maxnode, None)

    def _finalize(self, y):
        super()._finalize(y)
        # compute_regression_mse (src/rf_random_forest.cpp:4014-4058)
        s = self.acc_["oob_sum"]
        nout = self.acc_["nout"]
        oob = nout > 0
        pred = s.copy()
        pred[oob] = s[oob] / nout[oob].astype(np.float32)
        err = (self._y[oob] - pred[oob]).astype(np.float32)
        sq = (err * err).astype(np.float32)
        sse = np.add.accumulate(sq, dtype=np.float32)[-1] if len(sq) else np.float32(0)
        tot = int(oob.sum())
        self._oob_error = np.float32(sse / np.float32(tot)) if tot else np.float32(0)
        self._oob_pred = pred

    def get_oob_predictions(self):
        self._check()
        return self._oob_pred.copy()

    def get_oob_mse(self):
        return self.get_oob_error()

    def predict(self, X):
        """Mean of the trees' values (python/randomforest_py.cpp:1860-1869,
        src/rf_random_forest.cpp:3494-3590); training-size inputs are walked too."""
        self._check()
        return self._context().predict(np.ascontiguousarray(X, np.float32), 0)


class RandomForestUnsupervised(_Classifying):
    _TASK = A.TASK_UNSUPERVISED
    _task = A.TASK_UNSUPERVISED

    def __init__(self, nsample=1000, ntree=100, mdim=10, maxcat=10, mtry=0, maxnode=0,
                 minndsize=1, ncsplit=25, ncmax=25, iseed=12345, compute_proximity=True,
                 compute_importance=True, **kw):
        kw.setdefault("rank", 100)  # python/randomforest_py.cpp:5934-5974 defaults
        super().__init__(nsample=nsample, ntree=ntree, mdim=mdim, maxcat=maxcat, mtry=mtry,
                         maxnode=maxnode, minndsize=minndsize, ncsplit=ncsplit, ncmax=ncmax,
                         iseed=iseed, compute_proximity=compute_proximity,
                         compute_importance=compute_importance, **kw)

    def _resolve_mtry_ctor(self, mtry):
        return mtry  # 0 is resolved at fit time (setup_unsupervised_task)

    def fit(self, X, sample_weights=None):
        X = np.ascontiguousarray(X, dtype=np.float32)
        n, p = X.shape
        mtry = self._mtry if self._mtry > 0 else max(1, _isqrt_f32(p))
        maxnode = calculate_maxnode(2 * n, self.minndsize)  # src/rf_random_forest.cpp:1106
        self._fit(X, None, None, A.TASK_UNSUPERVISED, mtry, maxnode, None)

    def _finalize(self, y):
        super()._finalize(y)
        n2 = self.n_rows_
        labels = np.zeros(n2, np.int32)
        labels[: n2 // 2] = 1
        self._class_error_and_preds(labels)
