"""Proximity-based imputation (the reference's rfx_impute_proximity, python/rfx_impute.py:
596-793) with the forests and the fill rounds on the device.

Each iteration fits an unsupervised forest on the current matrix (proximity over the real
rows), then fills every originally-missing cell from the finished proximity row
(rfx_impute_round_ex: proximity-weighted mean for continuous columns, proximity-weighted mode
for categorical ones, numpy's summation order kept; or with aggregation 'median' the median
and the most frequent value; with top_k only the top_k rows by proximity), and stops early
when the summed change falls below 1e-6.  top_k keeps equal proximities in row order (the
reference's np.argsort leaves their order to numpy's sort implementation).
"""
from __future__ import annotations

import numpy as np

from . import _abi as A


def _encode(X):
    """Numeric float32 matrix, the mask of string-encoded columns and their encoders
    (strings -> 0-based codes in sorted label order, NaN kept; rfx_impute.py:142-237)."""
    try:
        import pandas as pd
    except ImportError:  # pragma: no cover
        pd = None
    if pd is not None and isinstance(X, pd.DataFrame):
        out = np.empty(X.shape, np.float32)
        auto = np.zeros(X.shape[1], bool)
        enc = {}
        for j in range(X.shape[1]):
            s = X.iloc[:, j]
            if s.dtype == "category" or s.dtype == object:
                cat = pd.Categorical(s)
                codes = cat.codes.astype(np.float32)
                codes[codes == -1] = np.nan
                out[:, j] = codes
                enc[j] = np.asarray(cat.categories)
                auto[j] = True
            elif s.dtype == bool:
                out[:, j] = s.astype(np.float32).values
                enc[j] = np.array([False, True])
                auto[j] = True
            else:
                out[:, j] = np.asarray(s.values, np.float32)
        return out, auto, enc
    arr = np.asarray(X)
    if arr.dtype == object:
        rows, cols = arr.shape
        out = np.empty((rows, cols), np.float32)
        auto = np.zeros(cols, bool)
        enc = {}

        def missing(v):
            return v is None or (isinstance(v, float) and np.isnan(v))

        for j in range(cols):
            col = arr[:, j]
            if any(isinstance(v, str) for v in col if not missing(v)):
                labels = sorted({v for v in col if not missing(v)})
                pos = {lab: k for k, lab in enumerate(labels)}
                out[:, j] = [np.nan if missing(v) else pos[v] for v in col]
                enc[j] = np.array(labels)
                auto[j] = True
            else:
                out[:, j] = [np.nan if v is None else float(v) for v in col]
        return out, auto, enc
    return np.asarray(X, np.float32), np.zeros(arr.shape[1], bool), {}


def _categorical_mask(categorical_features, p):
    if categorical_features is None:
        return None
    c = np.asarray(categorical_features)
    if c.dtype == bool:
        if c.shape != (p,):
            raise ValueError(f"categorical_features bool array length {len(c)} != n_features {p}")
        return c
    if np.issubdtype(c.dtype, np.integer):
        m = np.zeros(p, bool)
        m[c] = True
        return m
    raise TypeError("categorical_features must be a bool array or integer index array, "
                    f"got dtype={c.dtype}")


def _detect_categorical(X, max_unique):
    out = np.zeros(X.shape[1], bool)
    for j in range(X.shape[1]):
        v = X[:, j][~np.isnan(X[:, j])]
        if len(v):
            out[j] = len(np.unique(v)) <= max_unique and np.allclose(v, np.round(v))
    return out


def _rough_fill(X, is_cat):
    """Median (continuous) / mode (categorical) of the observed values (na.roughfix)."""
    Y = X.copy()
    for j in range(X.shape[1]):
        miss = np.isnan(Y[:, j])
        if not miss.any():
            continue
        v = Y[~miss, j]
        if len(v) == 0:
            Y[miss, j] = 0
        elif is_cat[j]:
            vals, counts = np.unique(v, return_counts=True)
            Y[miss, j] = vals[np.argmax(counts)]
        else:
            Y[miss, j] = np.median(v)
    return Y


def rfx_impute_proximity(X, ntree=100, n_iterations=5, use_gpu=True, categorical_features=None,
                         maxcat=10, show_progress=False, iseed=42, top_k=None, aggregation="mean",
                         nodesize=5, mtry=0, n_trees=None, seed=None, verbose=None,
                         max_categorical_unique=None, device=0, **rf_kwargs):
    """Returns (X_imputed float32, info) like the reference."""
    from .forest import RandomForestUnsupervised
    ntree = n_trees if n_trees is not None else ntree
    iseed = seed if seed is not None else iseed
    show_progress = verbose if verbose is not None else show_progress
    maxcat = max_categorical_unique if max_categorical_unique is not None else maxcat
    if aggregation not in ("mean", "weighted_mean", "median"):
        raise ValueError(f"Unknown aggregation: {aggregation}")
    if top_k is not None and int(top_k) < 0:
        raise ValueError("top_k must be None or >= 0")
    X, auto_cat, encoders = _encode(X)
    n, p = X.shape
    missing = np.isnan(X)
    n_missing = int(missing.sum())
    if n_missing == 0:
        return X.copy(), {"n_missing": 0, "encoders": encoders}
    cat = _categorical_mask(categorical_features, p)
    if cat is None:
        cat = _detect_categorical(X, maxcat)
    cat = cat | auto_cat
    Xi = _rough_fill(X, cat)
    auto_mtry = mtry if mtry > 0 else max(1, int(np.sqrt(p)))
    # cells in the reference's visiting order (column-major) and sorted by row for the device
    jj, ii = np.nonzero(missing.T)
    order = np.lexsort((jj, ii))
    cells = np.ascontiguousarray(np.stack([ii[order], jj[order]], axis=1).astype(np.int32))
    miss_cm = np.ascontiguousarray(missing.T.astype(np.uint8))
    cat_u8 = np.ascontiguousarray(cat.astype(np.uint8))
    it = 0
    timing = []
    import time
    for it in range(n_iterations):
        t0 = time.perf_counter()
        kw = dict(ntree=ntree, mtry=auto_mtry, nodesize=nodesize, iseed=iseed, use_gpu=use_gpu,
                  compute_proximity=True, compute_importance=False, show_progress=False)
        kw.update(rf_kwargs)
        model = RandomForestUnsupervised(prox_rows=n, device=device, **kw)
        model.fit(Xi)
        t1 = time.perf_counter()
        new = model._context().impute_round(np.ascontiguousarray(Xi.T), miss_cm, cat_u8, cells,
                                            top_k, aggregation)
        timing.append((t1 - t0, time.perf_counter() - t1))
        # apply, and the reference's change sum (float32 under numpy 2 scalar rules) in its
        # visiting order: columns ascending, rows ascending
        vals = np.full((n, p), np.nan, np.float32)
        vals[cells[:, 0], cells[:, 1]] = new
        nv = vals[ii, jj]
        ov = Xi[ii, jj]
        ok = ~np.isnan(nv)
        diffs = np.abs(nv[ok] - ov[ok]).astype(np.float32)
        changes = np.add.accumulate(diffs, dtype=np.float32)[-1] if len(diffs) else np.float32(0)
        Xi[ii[ok], jj[ok]] = nv[ok]
        if show_progress:
            print(f"    Iteration {it + 1}: total change {changes:.4f}")
        if changes < 1e-6:
            break
    info = {"n_missing_total": n_missing, "n_iterations": it + 1 if n_iterations > 0 else 0,
            "method": "proximity", "top_k": top_k, "aggregation": aggregation,
            "encoders": encoders, "timing_fit_fill_s": timing}
    return Xi, info


def rfx_impute_topk_mean(X, k=10, **kwargs):
    """Mean of the k rows most similar by proximity (python/rfx_impute.py:798-800)."""
    return rfx_impute_proximity(X, top_k=k, aggregation="mean", **kwargs)


def rfx_impute_topk_median(X, k=10, **kwargs):
    """Median of the k rows most similar by proximity (python/rfx_impute.py:803-805)."""
    return rfx_impute_proximity(X, top_k=k, aggregation="median", **kwargs)
