"""Bit-exact parity at the BASELINE configs' full data sizes (a few trees each, so the CPU
oracle finishes in seconds), plus forest-level invariants on a longer device run."""
import numpy as np
import pytest

import oracle
from _helpers import compare_fit, gpu_fit

pytestmark = pytest.mark.gpu


def config1_data(n=200_000, p=50, seed=20261201 + 1):
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1.0, 1.0, size=(n, p)).astype(np.float32)
    y = np.sin(3.0 * X[:, :10]).sum(axis=1) + 0.5 * X[:, 10] * X[:, 11]
    return X, (y + rng.normal(0.0, 0.1, size=n)).astype(np.float32)


def config0_data(n=10_000, p=20, seed=20261201 + 0):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, p)).astype(np.float32)
    w = rng.normal(size=p)
    y = (rng.random(n) < 1.0 / (1.0 + np.exp(-(X @ w)))).astype(np.int32)
    return X, y


def test_config1_full_size_two_trees():
    X, y = config1_data()
    M = oracle.maxnode(len(y), 5, 0)
    g = gpu_fit(1, X, y, ntree=2, mtry=16, minndsize=5, maxnode=M)
    o = oracle.fit(1, X, y, ntree=2, mtry=16, minndsize=5, maxnode=M)
    assert o["nnode"].min() > 1000
    compare_fit(g, o, 1)


@pytest.mark.parametrize("mode", ["push", "pull"])
def test_config0_full_size_with_proximity(mode, monkeypatch):
    monkeypatch.setenv("RFX_PROX_MODE", mode)
    X, y = config0_data()
    M = oracle.maxnode(len(y), 1, 0)
    g = gpu_fit(0, X, y, ntree=6, mtry=4, minndsize=1, maxnode=M, proximity=True)
    o = oracle.fit(0, X, y, ntree=6, mtry=4, minndsize=1, maxnode=M, proximity=True)
    compare_fit(g, o, 0, proximity=True)


def test_config1_forest_invariants():
    """64 trees at full size: every in-bag row lands in exactly one leaf, OOB counts and
    leaves agree with the bootstrap, and the trees are well formed."""
    X, y = config1_data()
    M = oracle.maxnode(len(y), 5, 0)
    T = 64
    g = gpu_fit(1, X, y, ntree=T, mtry=16, minndsize=5, maxnode=M, batch_trees=32)
    nin, st, tm, nn = g["nin"], g["nodestatus"], g["treemap"], g["nnode"]
    assert np.array_equal(g["nout"], (nin == 0).sum(0))
    assert np.array_equal(g["oob_leaf"] >= 0, nin == 0)
    for t in range(T):
        k = nn[t]
        assert 1 <= k <= M
        assert set(np.unique(st[t, :k])) <= {1, -1}
        assert np.all(st[t, k:] == 0)
        split = np.flatnonzero(st[t, :k] == 1)
        kids = np.sort(np.concatenate([tm[t, 2 * split], tm[t, 2 * split + 1]]))
        assert np.array_equal(kids, np.arange(1, k))  # every non-root node has one parent
        leaves = g["oob_leaf"][t][nin[t] == 0]
        assert np.all(st[t, leaves] == -1)
    assert np.array_equal(nin[0], oracle.bootstrap(len(y), 0))
