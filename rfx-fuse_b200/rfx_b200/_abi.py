"""ctypes binding of the C ABI in include/rfx_b200.h (librfx_b200.so, built in-tree).

The library is the only compute path: importing this module without the built library
raises, and there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librfx_b200.so")

RFX_OK = 0
ERRORS = {-1: "RFX_ERR_ARG", -2: "RFX_ERR_CUDA", -3: "RFX_ERR_OOM", -4: "RFX_ERR_UNSUPPORTED",
          -5: "RFX_ERR_STATE", -6: "RFX_ERR_DEVICE", -7: "RFX_ERR_CANCELLED"}
TASK_CLASSIFICATION, TASK_REGRESSION, TASK_UNSUPERVISED = 0, 1, 2

_pi = C.POINTER(C.c_int)
_pf = C.POINTER(C.c_float)
_pu8 = C.POINTER(C.c_uint8)


class FitParams(C.Structure):
    _fields_ = [(k, C.c_int) for k in (
        "task", "n", "p", "mtry", "minndsize", "maxnode", "iseed", "boot_seed", "nbins",
        "maxcat", "compute_importance", "compute_proximity", "prox_rows", "batch_trees",
        "keep_tree_oob", "lowrank_rank", "keep_forest", "keep_leaves", "keep_trees")]


class Inputs(C.Structure):
    _fields_ = [("X", _pf), ("y_class", _pi), ("y_reg", _pf), ("sample_weights", _pf),
                ("cat", _pi), ("classwt", _pf)]


class Trees(C.Structure):
    _fields_ = [("nodestatus", _pi), ("bestvar", _pi), ("xbestsplit", _pf), ("treemap", _pi),
                ("nodeclass", _pi), ("nnode", _pi), ("nodepred", _pf), ("tnodewt", _pf),
                ("nin", _pi), ("oob_leaf", _pi), ("tree_rr", _pf), ("tree_used", _pu8)]


class Accum(C.Structure):
    _fields_ = [("nclass", C.c_int), ("N", C.c_int), ("nout", _pi), ("votes", _pi),
                ("q", _pf), ("oob_sum", _pf), ("avimp", _pf), ("sqsd", _pf), ("labels", _pi)]


class Forest(C.Structure):
    _fields_ = [("task", C.c_int), ("ntree", C.c_int), ("maxnode", C.c_int), ("nclass", C.c_int),
                ("p", C.c_int), ("nodestatus", _pi), ("bestvar", _pi), ("xbestsplit", _pf),
                ("treemap", _pi), ("nodeclass", _pi), ("nodepred", _pf), ("cat", _pi),
                ("classwt", _pf)]


class Stats(C.Structure):
    _fields_ = [("kernel_launches", C.c_int64), ("hist_launches", C.c_int64),
                ("hist_ms", C.c_double), ("hist_bytes", C.c_double), ("levels", C.c_int64),
                ("trees", C.c_int64), ("prox_pair_updates", C.c_double), ("prox_ms", C.c_double),
                ("topk_ms", C.c_double), ("topk_tiles", C.c_int64), ("sketch_ms", C.c_double),
                ("sketch_bytes", C.c_double)]


SYMBOLS = (
    "rfx_last_error", "rfx_abi_version", "rfx_device_count", "rfx_cached_bytes", "rfx_empty_cache",
    "rfx_create", "rfx_destroy",
    "rfx_load", "rfx_grow", "rfx_results", "rfx_fit", "rfx_set_prox_buffer",
    "rfx_get_prox_buffer", "rfx_get_vote_buffers", "rfx_prox_finish", "rfx_prox_dense",
    "rfx_prox_finish_packed", "rfx_reset_forest", "rfx_set_progress", "rfx_get_trees",
    "rfx_oob_fold", "rfx_votes_to_q", "rfx_copy_to_host", "rfx_get_stream",
    "rfx_set_profiling", "rfx_get_stats", "rfx_reset_stats", "rfx_sync",
    "rfx_lowrank_build", "rfx_lowrank_factors", "rfx_lowrank_topk", "rfx_lowrank_product",
    "rfx_prox_apply", "rfx_lowrank_set_factors", "rfx_load_forest", "rfx_predict",
    "rfx_lowrank_topk_part", "rfx_impute_round", "rfx_impute_round_ex", "rfx_leaf_assignments", "rfx_leaf_index",
    "rfx_leaf_top_k_similar", "rfx_leaf_proximity", "rfx_predict_leaves",
    "rfx_predict_top_k_similar", "rfx_leaf_select_anchors", "rfx_leaf_outlier_scores",
    "rfx_rank_scores_desc", "rfx_predict_outlier_scores",
)

# int (*)(void* user, float* buf_dev, int64_t count): in-place sum over processes
REDUCE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int64)
# int (*)(void* user, int trees_done, int ntree): progress between batches; nonzero stops
PROGRESS_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.c_int)

_LIB = None


def rank_scores_desc(scores, k: int):
    """The reference's std::sort of (index, score) by score descending, first k."""
    L = load_library()
    sc = np.ascontiguousarray(scores, np.float32)
    kk = min(int(k), sc.shape[0])
    idx = np.zeros(max(kk, 1), np.int32)
    val = np.zeros(max(kk, 1), np.float32)
    check(L.rfx_rank_scores_desc(ptr(sc, _pf), sc.shape[0], kk, ptr(idx, _pi), ptr(val, _pf)))
    return idx[:kk], val[:kk]


def load_library(path: str = LIB_PATH):
    """Load librfx_b200.so and declare its signatures.  Raises if it is not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is not built; run `make -C rfx-fuse_b200` (sm_100a)")
    L = C.CDLL(path)
    vp = C.c_void_p
    L.rfx_last_error.restype = C.c_char_p
    L.rfx_abi_version.restype = C.c_int
    L.rfx_device_count.restype = C.c_int
    L.rfx_cached_bytes.restype = C.c_longlong
    L.rfx_cached_bytes.argtypes = [C.c_int]
    L.rfx_empty_cache.argtypes = [C.c_int]
    L.rfx_create.restype = vp
    L.rfx_create.argtypes = [C.c_int]
    L.rfx_destroy.argtypes = [vp]
    L.rfx_load.argtypes = [vp, C.POINTER(FitParams), C.POINTER(Inputs)]
    L.rfx_grow.argtypes = [vp, C.c_int, C.c_int, C.POINTER(Trees)]
    L.rfx_results.argtypes = [vp, C.POINTER(Accum)]
    L.rfx_fit.argtypes = [vp, C.POINTER(FitParams), C.POINTER(Inputs), C.c_int,
                          C.POINTER(Trees), C.POINTER(Accum)]
    L.rfx_set_prox_buffer.argtypes = [vp, vp, C.c_int64]
    L.rfx_get_prox_buffer.argtypes = [vp, C.POINTER(vp), C.POINTER(C.c_int64)]
    L.rfx_get_vote_buffers.argtypes = [vp, C.POINTER(vp), C.POINTER(vp)]
    L.rfx_prox_finish.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, vp]
    L.rfx_prox_dense.argtypes = [vp, C.c_int, C.c_int, _pf]
    L.rfx_prox_finish_packed.argtypes = [vp, vp, C.c_int64, C.c_int64, vp, C.c_int, vp]
    L.rfx_reset_forest.argtypes = [vp]
    L.rfx_get_trees.argtypes = [vp, C.c_int, C.c_int, C.POINTER(Trees)]
    L.rfx_set_progress.argtypes = [vp, PROGRESS_FN, vp]
    L.rfx_oob_fold.argtypes = [vp, vp]
    L.rfx_votes_to_q.argtypes = [vp, vp, _pf, C.c_int, C.c_int, vp]
    L.rfx_copy_to_host.argtypes = [vp, vp, vp, C.c_size_t]
    L.rfx_get_stream.argtypes = [vp, C.POINTER(vp)]
    L.rfx_set_profiling.argtypes = [vp, C.c_int]
    L.rfx_get_stats.argtypes = [vp, C.POINTER(Stats)]
    L.rfx_reset_stats.argtypes = [vp]
    L.rfx_sync.argtypes = [vp]
    L.rfx_lowrank_build.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_uint64, vp, REDUCE_FN, vp]
    L.rfx_lowrank_factors.argtypes = [vp, _pf, C.POINTER(C.c_int8), _pf, C.POINTER(C.c_int),
                                      C.POINTER(C.c_int)]
    L.rfx_lowrank_topk.argtypes = [vp, C.c_int, C.c_int, C.c_int, _pi, _pf]
    L.rfx_lowrank_product.argtypes = [vp, C.c_int, C.c_int, _pf]
    L.rfx_prox_apply.argtypes = [vp, vp, C.c_int, vp, vp]
    L.rfx_lowrank_set_factors.argtypes = [vp, C.POINTER(C.c_int8), _pf, C.c_int, C.c_int]
    L.rfx_load_forest.argtypes = [vp, C.POINTER(Forest)]
    L.rfx_impute_round.argtypes = [vp, _pf, _pu8, _pu8, C.c_int, C.c_int, _pi, C.c_int, _pf]
    L.rfx_impute_round_ex.argtypes = [vp, _pf, _pu8, _pu8, C.c_int, C.c_int, _pi, C.c_int,
                                      C.c_int, C.c_int, _pf]
    L.rfx_lowrank_topk_part.argtypes = [vp, C.c_int, C.c_int, C.c_int, _pi, _pi, _pf,
                                        C.POINTER(C.c_int)]
    L.rfx_predict.argtypes = [vp, _pf, C.c_int, C.c_int, _pi, _pf, _pf]
    _pi16 = C.POINTER(C.c_int16)
    L.rfx_leaf_assignments.argtypes = [vp, _pi16, _pi, _pi]
    L.rfx_leaf_index.argtypes = [vp]
    L.rfx_leaf_top_k_similar.argtypes = [vp, _pi, C.c_int, C.c_int, C.c_int, _pi, _pf, _pi]
    L.rfx_leaf_proximity.argtypes = [vp, C.c_int, C.c_int, _pf]
    L.rfx_predict_leaves.argtypes = [vp, _pf, C.c_int, C.c_int, _pi16]
    L.rfx_predict_top_k_similar.argtypes = [vp, _pf, C.c_int, C.c_int, C.c_int, _pi, _pf]
    L.rfx_leaf_select_anchors.argtypes = [vp, C.c_int, C.c_int, C.c_uint32, _pi, _pi]
    L.rfx_leaf_outlier_scores.argtypes = [vp, C.c_int, _pi, C.c_int, C.c_int, _pi, _pf, _pf]
    L.rfx_rank_scores_desc.argtypes = [_pf, C.c_int, C.c_int, _pi, _pf]
    L.rfx_predict_outlier_scores.argtypes = [vp, _pf, C.c_int, C.c_int, C.c_int, C.c_int, _pi, _pf]
    for name in ("rfx_load", "rfx_grow", "rfx_results", "rfx_fit", "rfx_set_prox_buffer",
                 "rfx_get_prox_buffer", "rfx_get_vote_buffers", "rfx_prox_finish",
                 "rfx_prox_finish_packed", "rfx_reset_forest", "rfx_set_progress", "rfx_get_trees",
                 "rfx_prox_dense", "rfx_oob_fold", "rfx_votes_to_q", "rfx_copy_to_host",
                 "rfx_get_stream", "rfx_set_profiling", "rfx_get_stats", "rfx_reset_stats",
                 "rfx_sync", "rfx_lowrank_build", "rfx_lowrank_factors", "rfx_lowrank_topk",
                 "rfx_lowrank_product", "rfx_prox_apply", "rfx_lowrank_set_factors",
                 "rfx_load_forest", "rfx_predict", "rfx_lowrank_topk_part",
                 "rfx_impute_round", "rfx_impute_round_ex", "rfx_leaf_assignments",
                 "rfx_leaf_index",
                 "rfx_leaf_top_k_similar", "rfx_leaf_proximity", "rfx_predict_leaves",
                 "rfx_predict_top_k_similar", "rfx_leaf_select_anchors",
                 "rfx_leaf_outlier_scores", "rfx_rank_scores_desc",
                 "rfx_predict_outlier_scores"):
        getattr(L, name).restype = C.c_int
    _LIB = L
    return L


class RfxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != RFX_OK:
        raise RfxError(rc, (load_library().rfx_last_error() or b"").decode(errors="replace"))


def ptr(a, t):
    return None if a is None else a.ctypes.data_as(t)


def cached_bytes(device: int = -1) -> int:
    """Bytes of device memory the library keeps from destroyed contexts for reuse (device -1:
    every device)."""
    return int(load_library().rfx_cached_bytes(int(device)))


def empty_cache(device: int = -1) -> None:
    """Free the device memory kept from destroyed contexts (device -1: every device), e.g.
    before another library in the process allocates."""
    check(load_library().rfx_empty_cache(int(device)))


class Context:
    """One CUDA device.  Owns the device copy of a loaded dataset and its accumulators."""

    def __init__(self, device: int = 0):
        L = load_library()
        self._lib = L
        h = L.rfx_create(int(device))
        if not h:
            raise RfxError(-2, (L.rfx_last_error() or b"").decode(errors="replace"))
        self.handle = C.c_void_p(h)
        self.device = device

    def close(self):
        if getattr(self, "handle", None):
            self._lib.rfx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load(self, prm: FitParams, inputs: Inputs):
        check(self._lib.rfx_load(self.handle, C.byref(prm), C.byref(inputs)))

    def grow(self, tree_begin: int, ntree: int, trees: Trees | None = None):
        check(self._lib.rfx_grow(self.handle, tree_begin, ntree,
                                 C.byref(trees) if trees is not None else None))

    def set_progress(self, fn=None):
        """fn(trees_done, ntree) -> truthy to stop, called between batches; None removes it."""
        if fn is None:
            self._progress = None
            check(self._lib.rfx_set_progress(self.handle, PROGRESS_FN(0), None))
            return

        def _cb(_user, done, total):
            try:
                return 1 if fn(int(done), int(total)) else 0
            except Exception:  # a failing callback stops the fit rather than crash it
                return 1
        self._progress = PROGRESS_FN(_cb)  # kept alive while registered
        check(self._lib.rfx_set_progress(self.handle, self._progress, None))

    def get_trees(self, tree_begin: int, count: int, trees: "Trees"):
        check(self._lib.rfx_get_trees(self.handle, int(tree_begin), int(count), C.byref(trees)))

    def reset_forest(self):
        check(self._lib.rfx_reset_forest(self.handle))

    def results(self, acc: Accum):
        check(self._lib.rfx_results(self.handle, C.byref(acc)))

    def prox_dense(self, r0: int, r1: int, out: np.ndarray):
        check(self._lib.rfx_prox_dense(self.handle, r0, r1, ptr(out, _pf)))

    def prox_buffer(self):
        p = C.c_void_p()
        n = C.c_int64()
        check(self._lib.rfx_get_prox_buffer(self.handle, C.byref(p), C.byref(n)))
        return p.value, n.value

    def set_prox_buffer(self, dev_ptr: int | None, length: int):
        check(self._lib.rfx_set_prox_buffer(self.handle, C.c_void_p(dev_ptr) if dev_ptr else None,
                                            C.c_int64(length)))

    def vote_buffers(self):
        a, b = C.c_void_p(), C.c_void_p()
        check(self._lib.rfx_get_vote_buffers(self.handle, C.byref(a), C.byref(b)))
        return a.value, b.value

    def prox_finish(self, upper_dev: int, nout_dev: int, R: int, r0: int, r1: int, out_dev: int):
        check(self._lib.rfx_prox_finish(self.handle, C.c_void_p(upper_dev), C.c_void_p(nout_dev),
                                        R, r0, r1, C.c_void_p(out_dev)))

    def prox_finish_packed(self, upper_dev: int, e0: int, count: int, nout_dev: int, R: int,
                           out_dev: int):
        check(self._lib.rfx_prox_finish_packed(self.handle, C.c_void_p(upper_dev), int(e0),
                                               int(count), C.c_void_p(nout_dev), int(R),
                                               C.c_void_p(out_dev)))

    def oob_fold(self, vec_dev: int):
        check(self._lib.rfx_oob_fold(self.handle, C.c_void_p(vec_dev)))

    def votes_to_q(self, votes_dev: int, classwt, N: int, nclass: int, q_dev: int):
        cw = None if classwt is None else np.ascontiguousarray(classwt, np.float32)
        check(self._lib.rfx_votes_to_q(self.handle, C.c_void_p(votes_dev), ptr(cw, _pf), N, nclass,
                                       C.c_void_p(q_dev)))

    def copy_to_host(self, dst: np.ndarray, src_dev: int):
        check(self._lib.rfx_copy_to_host(self.handle, dst.ctypes.data_as(C.c_void_p),
                                         C.c_void_p(src_dev), dst.nbytes))

    def stream(self) -> int:
        s = C.c_void_p()
        check(self._lib.rfx_get_stream(self.handle, C.byref(s)))
        return s.value or 0

    def set_profiling(self, on: bool):
        check(self._lib.rfx_set_profiling(self.handle, int(bool(on))))

    def stats(self) -> dict:
        s = Stats()
        check(self._lib.rfx_get_stats(self.handle, C.byref(s)))
        return {k: getattr(s, k) for k, _ in Stats._fields_}

    def reset_stats(self):
        check(self._lib.rfx_reset_stats(self.handle))

    def sync(self):
        check(self._lib.rfx_sync(self.handle))

    # ---- prediction ----
    def load_forest(self, task: int, trees: dict, cat, nclass: int = 1, classwt=None):
        """Put host tree arrays ([ntree][maxnode]: nodestatus, bestvar, xbestsplit, treemap
        (x2), nodeclass / nodepred) on the device for predict()."""
        arr = {k: np.ascontiguousarray(trees[k]) for k in
               ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass", "nodepred")
               if trees.get(k) is not None}
        T, M = arr["nodestatus"].shape
        cat = np.ascontiguousarray(cat, np.int32)
        cw = None if classwt is None else np.ascontiguousarray(classwt, np.float32)
        f = Forest(task, T, M, nclass, cat.shape[0], ptr(arr["nodestatus"], _pi),
                   ptr(arr["bestvar"], _pi), ptr(arr["xbestsplit"], _pf), ptr(arr["treemap"], _pi),
                   ptr(arr.get("nodeclass"), _pi), ptr(arr.get("nodepred"), _pf), ptr(cat, _pi),
                   ptr(cw, _pf))
        check(self._lib.rfx_load_forest(self.handle, C.byref(f)))

    def predict(self, X: np.ndarray, nclass: int = 0):
        """(classes int32 [n], proba float32 [n][nclass]) for a classification forest, or
        values float32 [n] for regression (nclass == 0)."""
        X = np.ascontiguousarray(X, np.float32)
        n, p = X.shape
        if nclass > 0:
            cls = np.zeros(n, np.int32)
            proba = np.zeros((n, nclass), np.float32)
            check(self._lib.rfx_predict(self.handle, ptr(X, _pf), n, p, ptr(cls, _pi),
                                        ptr(proba, _pf), None))
            return cls, proba
        val = np.zeros(n, np.float32)
        check(self._lib.rfx_predict(self.handle, ptr(X, _pf), n, p, None, None, ptr(val, _pf)))
        return val

    # ---- leaf assignments ----
    def leaf_assignments(self):
        """int16 [ntree][N] terminal node of every grown row in every tree."""
        T, N = C.c_int(0), C.c_int(0)
        check(self._lib.rfx_leaf_assignments(self.handle, None, C.byref(T), C.byref(N)))
        out = np.zeros((T.value, N.value), np.int16)
        check(self._lib.rfx_leaf_assignments(self.handle, out.ctypes.data_as(C.POINTER(C.c_int16)),
                                             None, None))
        return out

    def leaf_index(self):
        check(self._lib.rfx_leaf_index(self.handle))

    def leaf_top_k_similar(self, queries, k: int, exclude_self: bool = True):
        """Per query: (indices int32 [m], similarities float32 [m]), m <= k."""
        q = np.ascontiguousarray(queries, np.int32).reshape(-1)
        nq = q.shape[0]
        idx = np.zeros((nq, max(k, 1)), np.int32)
        sim = np.zeros((nq, max(k, 1)), np.float32)
        cnt = np.zeros(nq, np.int32)
        check(self._lib.rfx_leaf_top_k_similar(self.handle, ptr(q, _pi), nq, int(k),
                                               int(bool(exclude_self)), ptr(idx, _pi),
                                               ptr(sim, _pf), ptr(cnt, _pi)))
        return [(idx[i, :cnt[i]].copy(), sim[i, :cnt[i]].copy()) for i in range(nq)]

    def leaf_proximity(self, i: int, j: int) -> float:
        out = C.c_float(0.0)
        check(self._lib.rfx_leaf_proximity(self.handle, int(i), int(j), C.byref(out)))
        return out.value

    def predict_leaves(self, X: np.ndarray, ntree: int):
        X = np.ascontiguousarray(X, np.float32)
        n, p = X.shape
        out = np.zeros((n, ntree), np.int16)
        check(self._lib.rfx_predict_leaves(self.handle, ptr(X, _pf), n, p,
                                           out.ctypes.data_as(C.POINTER(C.c_int16))))
        return out

    def predict_top_k_similar(self, X: np.ndarray, k: int):
        X = np.ascontiguousarray(X, np.float32)
        n, p = X.shape
        idx = np.zeros((n, k), np.int32)
        sim = np.zeros((n, k), np.float32)
        check(self._lib.rfx_predict_top_k_similar(self.handle, ptr(X, _pf), n, p, int(k),
                                                  ptr(idx, _pi), ptr(sim, _pf)))
        return idx, sim

    def select_anchors(self, n_anchors: int, method: int, iseed: int):
        out = np.zeros(max(1, int(n_anchors)), np.int32)
        cnt = C.c_int(0)
        check(self._lib.rfx_leaf_select_anchors(self.handle, int(n_anchors), int(method),
                                                C.c_uint32(int(iseed) & 0xFFFFFFFF),
                                                ptr(out, _pi), C.byref(cnt)))
        return out[:cnt.value].copy()

    def outlier_scores(self, mode: int, anchors, n_anchors: int, labels, nrows: int):
        """(normalised scores, raw measures), float32 [nrows] each."""
        a = None if anchors is None else np.ascontiguousarray(anchors, np.int32)
        lab = None if labels is None else np.ascontiguousarray(labels, np.int32)
        sc = np.zeros(nrows, np.float32)
        raw = np.zeros(nrows, np.float32)
        check(self._lib.rfx_leaf_outlier_scores(self.handle, int(mode),
                                                None if a is None else ptr(a, _pi),
                                                0 if a is None else a.shape[0], int(n_anchors),
                                                None if lab is None else ptr(lab, _pi),
                                                ptr(sc, _pf), ptr(raw, _pf)))
        return sc, raw

    def predict_outlier_scores(self, X: np.ndarray, mode: int, n_anchors: int, classes=None):
        X = np.ascontiguousarray(X, np.float32)
        n, p = X.shape
        cl = None if classes is None else np.ascontiguousarray(classes, np.int32)
        out = np.zeros(n, np.float32)
        check(self._lib.rfx_predict_outlier_scores(self.handle, ptr(X, _pf), n, p, int(mode),
                                                   int(n_anchors),
                                                   None if cl is None else ptr(cl, _pi),
                                                   ptr(out, _pf)))
        return out

    # ---- imputation ----
    def impute_round(self, xc: np.ndarray, miss: np.ndarray, is_cat: np.ndarray, cells: np.ndarray,
                     top_k=None, aggregation="mean"):
        """New values of `cells` ([m, 2] (row, column), sorted by row) from this context's
        proximity; NaN = keep.  xc / miss are [p][n] (column-major).  top_k None or >= 0;
        aggregation 'mean' / 'weighted_mean' / 'median'."""
        agg = {"mean": 0, "weighted_mean": 0, "median": 1}.get(aggregation)
        if agg is None:
            raise ValueError(f"Unknown aggregation: {aggregation}")
        xc = np.ascontiguousarray(xc, np.float32)
        miss = np.ascontiguousarray(miss, np.uint8)
        is_cat = np.ascontiguousarray(is_cat, np.uint8)
        cells = np.ascontiguousarray(cells, np.int32)
        p, n = xc.shape
        out = np.zeros(cells.shape[0], np.float32)
        check(self._lib.rfx_impute_round_ex(self.handle, ptr(xc, _pf), ptr(miss, _pu8),
                                            ptr(is_cat, _pu8), n, p, ptr(cells, _pi),
                                            cells.shape[0], -1 if top_k is None else int(top_k),
                                            agg, ptr(out, _pf)))
        return out

    # ---- low-rank proximity ----
    def lowrank_build(self, rank: int, oversample: int = 16, power_iters: int = 1, seed: int = 0,
                      nout_dev: int | None = None, reduce=None):
        """Build the int8 factors.  ``reduce(dev_ptr, count)`` (optional) sums a device float
        buffer over the processes in place; it runs once per sketch pass."""
        cb = REDUCE_FN(0)
        if reduce is not None:
            def _cb(_user, buf, count):
                try:
                    reduce(int(buf), int(count))
                    return 0
                except Exception:  # reported as RFX_ERR_DEVICE by the library
                    return 1
            cb = REDUCE_FN(_cb)
        check(self._lib.rfx_lowrank_build(self.handle, int(rank), int(oversample),
                                          int(power_iters), C.c_uint64(seed & (2**64 - 1)),
                                          C.c_void_p(nout_dev) if nout_dev else None, cb, None))

    def lowrank_set_factors(self, q: np.ndarray, scale: np.ndarray):
        q = np.ascontiguousarray(q, np.int8)
        scale = np.ascontiguousarray(scale, np.float32)
        check(self._lib.rfx_lowrank_set_factors(self.handle, q.ctypes.data_as(C.POINTER(C.c_int8)),
                                                ptr(scale, _pf), q.shape[0], q.shape[1]))

    def lowrank_factors(self):
        """(A float32 [R, k] dequantised, q int8 [R, k], scale float32 [R])."""
        k, R = C.c_int(), C.c_int()
        check(self._lib.rfx_lowrank_factors(self.handle, None, None, None, C.byref(k), C.byref(R)))
        A = np.zeros((R.value, k.value), np.float32)
        q = np.zeros((R.value, k.value), np.int8)
        s = np.zeros(R.value, np.float32)
        check(self._lib.rfx_lowrank_factors(self.handle, ptr(A, _pf), q.ctypes.data_as(C.POINTER(C.c_int8)),
                                            ptr(s, _pf), C.byref(k), C.byref(R)))
        return A, q, s

    def lowrank_topk(self, k: int, r0: int, r1: int):
        idx = np.zeros((r1 - r0, k), np.int32)
        val = np.zeros((r1 - r0, k), np.float32)
        check(self._lib.rfx_lowrank_topk(self.handle, int(k), int(r0), int(r1), ptr(idx, _pi),
                                         ptr(val, _pf)))
        return idx, val

    def lowrank_topk_part(self, k: int, part: int, nparts: int):
        """(rows int32 [m], idx int32 [m, k], val float32 [m, k]) for one share of the rows."""
        m = C.c_int()
        check(self._lib.rfx_lowrank_topk_part(self.handle, int(k), int(part), int(nparts), None,
                                              None, None, C.byref(m)))
        rows = np.zeros(m.value, np.int32)
        idx = np.zeros((m.value, k), np.int32)
        val = np.zeros((m.value, k), np.float32)
        if m.value:
            check(self._lib.rfx_lowrank_topk_part(self.handle, int(k), int(part), int(nparts),
                                                  ptr(rows, _pi), ptr(idx, _pi), ptr(val, _pf),
                                                  C.byref(m)))
        return rows, idx, val

    def lowrank_product(self, r0: int, r1: int, R: int):
        out = np.zeros((r1 - r0, R), np.float32)
        check(self._lib.rfx_lowrank_product(self.handle, int(r0), int(r1), ptr(out, _pf)))
        return out

    def prox_apply(self, X_dev: int, ncols: int, Y_dev: int, nout_dev: int | None = None):
        check(self._lib.rfx_prox_apply(self.handle, C.c_void_p(X_dev), int(ncols),
                                       C.c_void_p(nout_dev) if nout_dev else None,
                                       C.c_void_p(Y_dev)))
