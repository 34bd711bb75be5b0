"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers of the hot path.

* ``librfx_oracle.so`` -- the CPU restatement (``rfx_oracle.cpp``) of the reference
  algorithm: bootstrap, quantile binning, histogram tree growth, OOB drop, permutation
  importance, proximity counts and finishprox.
* ``_ref/libref_harness.so`` -- the reference's own CPU implementation compiled from its
  unmodified sources (``Makefile`` target ``ref``), driven by ``ref_harness.cpp``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this
package, as the checker.  The product library never does.
"""
from __future__ import annotations

import ctypes as C
import glob
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_ORC = None
_REF = None

_i = C.c_int
_pi = C.POINTER(C.c_int)
_pf = C.POINTER(C.c_float)
_pd = C.POINTER(C.c_double)
_pu8 = C.POINTER(C.c_uint8)


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def reference_tree():
    """The reference source tree: $RFX_REFERENCE, else a directory named ``reference`` beside
    this repository; None when neither exists."""
    cand = os.environ.get("RFX_REFERENCE") or os.path.join(
        os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(cand) else None


def build(ref: bool = False) -> None:
    """Compile the oracle (and, when the reference tree is present, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    tree = reference_tree() if ref else None
    if tree:
        subprocess.run(["make", "-s", "-j8", "-C", HERE, "ref", "REF=" + tree], check=True)


class OrcParams(C.Structure):
    _fields_ = [(k, C.c_int) for k in (
        "task", "n", "p", "ntree", "mtry", "minndsize", "maxnode", "iseed", "boot_seed",
        "nbins", "compute_importance", "compute_proximity", "n_threads")]


class OrcOut(C.Structure):
    _fields_ = [("nclass", C.c_int), ("N", C.c_int),
                ("nodestatus", _pi), ("bestvar", _pi), ("xbestsplit", _pf), ("treemap", _pi),
                ("nodeclass", _pi), ("nnode", _pi), ("nodepred", _pf), ("tnodewt", _pf),
                ("nin_all", _pi), ("nodextr_all", _pi), ("nout", _pi), ("votes", _pi),
                ("q_raw", _pf), ("oob_sum", _pf), ("tree_rr", _pf), ("avimp", _pf),
                ("sqsd", _pf), ("prox_pairs", _pi), ("prox_final", _pd), ("oob_error", _pf),
                ("oob_pred", _pf)]


def lib():
    global _ORC
    if _ORC is None:
        path = os.path.join(HERE, "librfx_oracle.so")
        if not os.path.exists(path):
            build()
        _ORC = C.CDLL(path)
    return _ORC


def maxnode(n, minndsize, user_maxnode=0):
    return lib().orc_maxnode(n, minndsize, user_maxnode)


def bootstrap(n, tree_id, seed_base=12345, sample_weights=None):
    nin = np.zeros(n, np.int32)
    sw = None if sample_weights is None else np.ascontiguousarray(sample_weights, np.float32)
    lib().orc_bootstrap(n, tree_id, seed_base, _p(sw, _pf), _p(nin, _pi))
    return nin


def binning(X, cat=None, nbins=256):
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    edges = np.zeros((p, nbins + 1), np.float32)
    nb = np.zeros(p, np.int32)
    kind = np.zeros(p, np.int32)
    xb = np.zeros((n, p), np.uint8)
    c = None if cat is None else np.ascontiguousarray(cat, np.int32)
    lib().orc_binning(_p(X, _pf), n, p, _p(c, _pi), nbins, _p(edges, _pf), _p(nb, _pi),
                      _p(kind, _pi), _p(xb, _pu8))
    return edges, nb, kind, xb


def permutation(n, seed=42):
    perm = np.zeros(n, np.int32)
    lib().orc_permutation(n, C.c_uint32(seed), _p(perm, _pi))
    return perm


def synthetic(X, iseed=12345):
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    out = np.zeros((2 * n, p), np.float32)
    lib().orc_synthetic(_p(X, _pf), n, p, iseed, _p(out, _pf))
    return out


def finishprox(nout, pairs):
    N = len(nout)
    out = np.zeros((N, N), np.float64)
    lib().orc_finishprox(N, _p(np.ascontiguousarray(nout, np.int32), _pi),
                         _p(np.ascontiguousarray(pairs, np.int32), _pi), _p(out, _pd))
    return out


def predict(task, trees, X, nclass, cat, classwt=None):
    """orc_predict on the tree arrays of a fit (dict with nodestatus, bestvar, xbestsplit,
    treemap, nodeclass, nodepred).  Returns (cls, proba) for classification, pred for
    regression."""
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    T, M = trees["nodestatus"].shape
    cat = np.ascontiguousarray(cat, np.int32)
    cw = None if classwt is None else np.ascontiguousarray(classwt, np.float32)
    arr = {k: np.ascontiguousarray(trees[k]) for k in
           ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass", "nodepred")}
    cls = np.zeros(n, np.int32)
    proba = np.zeros((n, max(nclass, 1)), np.float32)
    reg = np.zeros(n, np.float32)
    lib().orc_predict(task, T, M, nclass, p, _p(cat, _pi), _p(cw, _pf),
                      _p(arr["nodestatus"], _pi), _p(arr["bestvar"], _pi),
                      _p(arr["xbestsplit"], _pf), _p(arr["treemap"], _pi),
                      _p(arr["nodeclass"], _pi), _p(arr["nodepred"], _pf), _p(X, _pf), n,
                      _p(cls, _pi), _p(proba, _pf), _p(reg, _pf))
    return reg if task == 1 else (cls, proba)


def fit(task, X, y=None, *, ntree, mtry, minndsize, maxnode, iseed=12345, nbins=256,
        sample_weights=None, cat=None, classwt=None, importance=True, proximity=False,
        dump_trees=True):
    """Run the oracle fit.  ``task``: 0 classification, 1 regression, 2 unsupervised.

    ``maxnode`` is the effective node cap (as resolved by the estimator wrapper).
    Returns a dict of numpy arrays.
    """
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    N = 2 * n if task == 2 else n
    prm = OrcParams(task, n, p, ntree, mtry, minndsize, maxnode, iseed, 12345, nbins,
                    int(importance), int(proximity), 0)
    ycls = np.ascontiguousarray(y, np.int32) if task == 0 else None
    yreg = np.ascontiguousarray(y, np.float32) if task == 1 else None
    ncl = len(np.unique(ycls)) if task == 0 else (2 if task == 2 else 1)
    r = {
        "nodestatus": np.zeros((ntree, maxnode), np.int32),
        "bestvar": np.zeros((ntree, maxnode), np.int32),
        "xbestsplit": np.zeros((ntree, maxnode), np.float32),
        "treemap": np.zeros((ntree, 2 * maxnode), np.int32),
        "nodeclass": np.zeros((ntree, maxnode), np.int32),
        "nnode": np.zeros(ntree, np.int32),
        "nodepred": np.zeros((ntree, maxnode), np.float32),
        "tnodewt": np.zeros((ntree, maxnode), np.float32),
        "nin": np.zeros((ntree, N), np.int32) if dump_trees else None,
        "nodextr": np.zeros((ntree, N), np.int32) if dump_trees else None,
        "nout": np.zeros(N, np.int32),
        "votes": np.zeros((N, ncl), np.int32),
        "q": np.zeros((N, ncl), np.float32),
        "oob_sum": np.zeros(N, np.float32),
        "tree_rr": np.zeros((ntree, p), np.float32),
        "avimp": np.zeros(p, np.float32),
        "sqsd": np.zeros(p, np.float32),
        "prox_pairs": np.zeros((N, N), np.int32) if proximity else None,
        "prox": np.zeros((N, N), np.float64) if proximity else None,
        "oob_error": np.zeros(1, np.float32),
        "oob_pred": np.zeros(N, np.float32),
    }
    o = OrcOut(0, 0, *[_p(r[k], t) for k, t in (
        ("nodestatus", _pi), ("bestvar", _pi), ("xbestsplit", _pf), ("treemap", _pi),
        ("nodeclass", _pi), ("nnode", _pi), ("nodepred", _pf), ("tnodewt", _pf),
        ("nin", _pi), ("nodextr", _pi), ("nout", _pi), ("votes", _pi), ("q", _pf),
        ("oob_sum", _pf), ("tree_rr", _pf), ("avimp", _pf), ("sqsd", _pf),
        ("prox_pairs", _pi), ("prox", _pd), ("oob_error", _pf), ("oob_pred", _pf))])
    sw = None if sample_weights is None else np.ascontiguousarray(sample_weights, np.float32)
    c = None if cat is None else np.ascontiguousarray(cat, np.int32)
    cw = None if classwt is None else np.ascontiguousarray(classwt, np.float32)
    lib().orc_fit(C.byref(prm), _p(X, _pf), _p(ycls, _pi), _p(yreg, _pf), _p(sw, _pf),
                  _p(c, _pi), _p(cw, _pf), C.byref(o))
    r["nclass"] = o.nclass
    r["oob_error"] = float(r["oob_error"][0])
    return r


# ---------------------------------------------------------------------------------------
# The reference itself (oracle/_ref), available only where it was compiled.
# ---------------------------------------------------------------------------------------
class RefOut(C.Structure):
    _fields_ = [("nclass", C.c_int), ("maxnode", C.c_int), ("nsample_total", C.c_int),
                ("mtry", C.c_int),
                ("nodestatus", _pi), ("bestvar", _pi), ("xbestsplit", _pf), ("treemap", _pi),
                ("nodeclass", _pi), ("nnode", _pi), ("nodepred", _pf), ("tnodewt", _pf),
                ("nin_all", _pi), ("nodextr_all", _pi), ("nout", _pi), ("q_raw", _pf),
                ("oob_pred", _pf), ("avimp", _pf), ("sqsd", _pf), ("prox_raw", _pd),
                ("prox_final", _pd), ("oob_error", _pf), ("X_expanded", _pf)]


def ref_dir():
    return os.path.join(HERE, "_ref")


def ref_available():
    return os.path.exists(os.path.join(ref_dir(), "libref_harness.so"))


_REF_STOCK = None


def ref_lib(stock: bool = False):
    """The reference harness; ``stock``: the build with the reference's stock flags only
    (``make ref-stock``: GCC free to contract into FMAs) instead of -ffp-contract=off."""
    global _REF, _REF_STOCK
    if stock:
        if _REF_STOCK is None:
            _REF_STOCK = C.CDLL(os.path.join(HERE, "_ref_stock", "libref_harness.so"))
        return _REF_STOCK
    if _REF is None:
        _REF = C.CDLL(os.path.join(ref_dir(), "libref_harness.so"))
    return _REF


def ref_module():
    """Import the reference Python module RFXFuse built under oracle/_ref."""
    import importlib
    import sys
    d = ref_dir()
    if not glob.glob(os.path.join(d, "RFXFuse*.so")):
        raise ImportError("oracle/_ref/RFXFuse is not built")
    if d not in sys.path:
        sys.path.insert(0, d)
    return importlib.import_module("RFXFuse")


def ref_bootstrap(n, tree_id, sample_weights=None):
    nin = np.zeros(n, np.int32)
    sw = None if sample_weights is None else np.ascontiguousarray(sample_weights, np.float32)
    ref_lib().ref_bootstrap(n, tree_id, _p(sw, _pf), _p(nin, _pi))
    return nin


def ref_binning(X, cat=None, nbins=256):
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    edges = np.zeros((p, nbins + 1), np.float32)
    nb = np.zeros(p, np.int32)
    kind = np.zeros(p, np.int32)
    xb = np.zeros((n, p), np.uint8)
    c = None if cat is None else np.ascontiguousarray(cat, np.int32)
    ref_lib().ref_binning(_p(X, _pf), n, p, _p(c, _pi), nbins, _p(edges, _pf), _p(nb, _pi),
                          _p(kind, _pi), _p(xb, _pu8))
    return edges, nb, kind, xb


def ref_fit(task, X, y=None, *, ntree, mtry, minndsize, maxnode=0, iseed=12345, nbins=256,
            sample_weights=None, cat=None, classwt=None, importance=True, proximity=False,
            stock=False):
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    L = ref_lib(stock)
    M = L.ref_effective_maxnode(task, n, minndsize, maxnode)
    N = 2 * n if task == 2 else n
    ycls = np.ascontiguousarray(y, np.int32) if task == 0 else None
    yreg = np.ascontiguousarray(y, np.float32) if task == 1 else None
    ncl = len(np.unique(ycls)) if task == 0 else (2 if task == 2 else 1)
    r = {
        "nodestatus": np.zeros((ntree, M), np.int32),
        "bestvar": np.zeros((ntree, M), np.int32),
        "xbestsplit": np.zeros((ntree, M), np.float32),
        "treemap": np.zeros((ntree, 2 * M), np.int32),
        "nodeclass": np.zeros((ntree, M), np.int32),
        "nnode": np.zeros(ntree, np.int32),
        "nodepred": np.zeros((ntree, M), np.float32),
        "tnodewt": np.zeros((ntree, M), np.float32),
        "nin": np.zeros((ntree, N), np.int32),
        "nodextr": np.zeros((ntree, N), np.int32),
        "nout": np.zeros(N, np.int32),
        "q": np.zeros((N, ncl), np.float32),
        "oob_pred": np.zeros(N, np.float32),
        "avimp": np.zeros(p, np.float32),
        "sqsd": np.zeros(p, np.float32),
        "prox_raw": np.zeros((N, N), np.float64) if proximity else None,
        "prox": np.zeros((N, N), np.float64) if proximity else None,
        "oob_error": np.zeros(1, np.float32),
        "X_expanded": np.zeros((N, p), np.float32) if task == 2 else None,
    }
    o = RefOut(0, 0, 0, 0, *[_p(r[k], t) for k, t in (
        ("nodestatus", _pi), ("bestvar", _pi), ("xbestsplit", _pf), ("treemap", _pi),
        ("nodeclass", _pi), ("nnode", _pi), ("nodepred", _pf), ("tnodewt", _pf),
        ("nin", _pi), ("nodextr", _pi), ("nout", _pi), ("q", _pf), ("oob_pred", _pf),
        ("avimp", _pf), ("sqsd", _pf), ("prox_raw", _pd), ("prox", _pd),
        ("oob_error", _pf), ("X_expanded", _pf))])
    sw = None if sample_weights is None else np.ascontiguousarray(sample_weights, np.float32)
    c = None if cat is None else np.ascontiguousarray(cat, np.int32)
    cw = None if classwt is None else np.ascontiguousarray(classwt, np.float32)
    L.ref_fit(task, _p(X, _pf), _p(ycls, _pi), _p(yreg, _pf), _p(sw, _pf), _p(c, _pi),
              _p(cw, _pf), n, p, ntree, mtry, minndsize, maxnode, iseed, nbins,
              int(importance), int(proximity), C.byref(o))
    r["nclass"], r["maxnode"], r["mtry"] = o.nclass, o.maxnode, o.mtry
    r["oob_error"] = float(r["oob_error"][0])
    return r
