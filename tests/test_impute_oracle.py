"""The CPU restatement of the imputation fill (oracle/impute_fill.py) against the reference's
rfx_impute_proximity, every aggregation and top_k, on the golden imputation data.  The
reference's forests come from its own compiled module (oracle/_ref); skipped without it.

With the reference's own np.argsort (sort_kind=None) the restated loop reproduces the
reference bit for bit, so the stable tie order that the device uses is the only difference
at a top_k cut."""
import importlib
import os
import sys

import numpy as np
import pytest

import oracle
from oracle.impute_fill import fill

HERE = os.path.dirname(os.path.abspath(__file__))


def _reference():
    tree = oracle.reference_tree()
    if tree is None or not oracle.ref_available():
        pytest.skip("reference sources / oracle/_ref not present")
    sys.path.insert(0, oracle.ref_dir())
    sys.path.insert(0, os.path.join(tree, "python"))
    return importlib.import_module("rfx_impute"), oracle.ref_module()


def _loop(ri, R, X, top_k, aggregation, sort_kind, n_iterations=2):
    """rfx_impute_proximity (python/rfx_impute.py:689-779) with the fill restated."""
    Xe, auto, _ = ri._auto_encode(X)
    n, p = Xe.shape
    miss = np.isnan(Xe)
    cat = ri._detect_categorical(Xe, 10) | auto
    Xi = ri._rough_impute(Xe, cat)
    for _ in range(n_iterations):
        m = R.RandomForestUnsupervised(ntree=25, mtry=max(1, int(np.sqrt(p))), nodesize=5,
                                       iseed=42, use_gpu=False, compute_proximity=True,
                                       compute_importance=False, show_progress=False,
                                       minndsize=1)
        m.fit(Xi)
        prox = m.get_proximity_matrix()[:n, :n]
        jj, ii = np.nonzero(miss.T)
        cells = np.stack([ii, jj], 1)
        new = fill(prox, Xi, miss, cat, cells, top_k, aggregation, sort_kind)
        change = 0.0
        for (i, j), v in zip(cells, new):
            if not np.isnan(v):
                change += abs(v - Xi[i, j])
                Xi[i, j] = v
        if change < 1e-6:
            break
    return Xi


@pytest.mark.parametrize("top_k,aggregation", [(None, "mean"), (None, "median"), (10, "mean"),
                                               (10, "median"), (3, "weighted_mean")])
def test_fill_restatement_reproduces_reference(top_k, aggregation):
    ri, R = _reference()
    sys.path.insert(0, os.path.join(HERE, "golden"))
    from make_golden import impute_data
    X = impute_data()
    want, _ = ri.rfx_impute_proximity(X.copy(), ntree=25, n_iterations=2, use_gpu=False,
                                      iseed=42, minndsize=1, top_k=top_k,
                                      aggregation=aggregation)
    got = _loop(ri, R, X.copy(), top_k, aggregation, None)
    assert np.array_equal(np.asarray(got, np.float32).view(np.uint32),
                          np.asarray(want, np.float32).view(np.uint32))


def test_imputation_rejects_bad_aggregation_and_top_k():
    """Argument checks run before any device work (python/rfx_impute.py raises ValueError
    for an unknown aggregation)."""
    import rfx_b200
    X = np.array([[1.0, np.nan], [2.0, 3.0], [np.nan, 4.0]], np.float32)
    with pytest.raises(ValueError):
        rfx_b200.rfx_impute_proximity(X, aggregation="mode")
    with pytest.raises(ValueError):
        rfx_b200.rfx_impute_proximity(X, top_k=-1)
