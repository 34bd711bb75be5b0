"""The process-wide cache of device blocks from destroyed contexts: a new fit reuses them and
gets the same forest; empty_cache frees them and the next fit allocates afresh."""
import gc

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _fit(X, y):
    import rfx_b200
    est = rfx_b200.RandomForestRegressor(nsample=X.shape[0], ntree=12, mtry=3, minndsize=5)
    est.fit(X, y)
    return est.get_oob_predictions(), est.feature_importances_()


def test_fits_through_cached_blocks_agree():
    import rfx_b200
    rng = np.random.default_rng(3)
    X = rng.normal(size=(3000, 8)).astype(np.float32)
    y = (X[:, 0] - 2 * X[:, 1] + 0.1 * rng.normal(size=3000)).astype(np.float32)
    rfx_b200.empty_cache()
    first = _fit(X, y)
    gc.collect()  # the estimator's context is destroyed: its blocks go to the cache
    assert rfx_b200.cached_bytes() > 0
    second = _fit(X, y)  # runs on cached blocks
    gc.collect()
    rfx_b200.empty_cache()
    assert rfx_b200.cached_bytes() == 0
    third = _fit(X, y)  # fresh allocations
    for a, b in ((first, second), (first, third)):
        assert np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32))
        assert np.array_equal(np.asarray(a[1]).view(np.uint32), np.asarray(b[1]).view(np.uint32))
