"""Device path (librfx_b200.so through the C ABI) vs the CPU oracle, bit for bit.

Tree structure, split variables and values, node classes / predictions, bootstrap counts,
OOB leaves, OOB votes and vote sums, OOB prediction sums, per-tree importance and its
tree-order sums, and proximity counts must all be identical to the oracle's (which is
itself pinned to the reference build by tests/test_oracle_golden.py).
"""
import numpy as np
import pytest

import oracle
from _helpers import compare_fit, gpu_fit, synth

pytestmark = pytest.mark.gpu


def both(task, X, y, **kw):
    n = X.shape[0]
    M = kw.pop("maxnode", None)
    if M is None:
        M = oracle.maxnode(2 * n if task == 2 else n, kw["minndsize"], 0)
    gkw = {k: v for k, v in kw.items() if k not in ()}
    okw = {k: v for k, v in kw.items() if k not in ("batch_trees", "tree_chunks")}
    g = gpu_fit(task, X, y, maxnode=M, **gkw)
    o = oracle.fit(task, X, y, maxnode=M, **okw)
    return g, o


@pytest.mark.parametrize("mode", ["push", "pull", "auto"])
def test_classification_proximity(mode, monkeypatch):
    # counts pushed per pair (atomics) or pulled per 128x128 tile (leaf-code compares)
    monkeypatch.setenv("RFX_PROX_MODE", mode)
    X, y = synth("class", 1500, 12, 1)
    g, o = both(0, X, y, ntree=7, mtry=3, minndsize=1, proximity=True)
    compare_fit(g, o, 0, proximity=True)


def test_multiclass_classwt_minnd2():
    X, y = synth("multiclass", 2000, 10, 2)
    g, o = both(0, X, y, ntree=5, mtry=3, minndsize=2, classwt=[0.1, 0.4, 0.7, 1.0])
    compare_fit(g, o, 0)


def test_regression_importance():
    X, y = synth("regr", 3000, 12, 3)
    g, o = both(1, X, y, ntree=6, mtry=4, minndsize=5)
    compare_fit(g, o, 1)


def test_regression_few_bins_and_node_cap():
    X, y = synth("regr", 2500, 8, 4)
    g, o = both(1, X, y, ntree=5, mtry=3, minndsize=2, nbins=16, maxnode=151)
    compare_fit(g, o, 1)


@pytest.mark.parametrize("mode", ["push", "pull"])
def test_unsupervised_proximity(mode, monkeypatch):
    monkeypatch.setenv("RFX_PROX_MODE", mode)
    X, _ = synth("gmm", 600, 8, 5)
    g, o = both(2, X, None, ntree=4, mtry=3, minndsize=1, proximity=True)
    compare_fit(g, o, 2, proximity=True)


def test_weighted_bootstrap():
    X, y = synth("class", 1200, 6, 6)
    w = np.random.default_rng(6).uniform(0.1, 3.0, size=1200).astype(np.float32)
    g, o = both(0, X, y, ntree=5, mtry=2, minndsize=1, sample_weights=w)
    compare_fit(g, o, 0)


def test_batches_and_calls_accumulate_in_tree_order():
    X, y = synth("regr", 1800, 6, 7)
    g, o = both(1, X, y, ntree=7, mtry=2, minndsize=3, batch_trees=3, tree_chunks=[3, 4])
    compare_fit(g, o, 1)


def test_binary_categorical_and_ties():
    rng = np.random.default_rng(8)
    n = 1600
    X = np.empty((n, 6), np.float32)
    X[:, 0] = rng.integers(0, 2, n)                 # binary
    X[:, 1] = rng.integers(0, 6, n)                 # categorical (6 levels)
    X[:, 2] = np.round(rng.normal(size=n), 1)       # many ties
    X[:, 3] = rng.normal(size=n)
    X[:, 4] = 3.0                                   # constant
    X[:, 5] = rng.integers(0, 2, n) * 5.0 + 1.0     # binary, wide gap
    y = ((X[:, 1] > 2) ^ (X[:, 3] > 0.3)).astype(np.int32)
    cat = np.array([1, 6, 1, 1, 1, 1], np.int32)
    g, o = both(0, X, y, ntree=5, mtry=3, minndsize=1, cat=cat)
    compare_fit(g, o, 0)


def test_regression_quantized_targets_and_values():
    rng = np.random.default_rng(9)
    n = 2200
    X = np.round(rng.uniform(-1, 1, size=(n, 7)), 2).astype(np.float32)
    y = (np.round(X[:, 0] * 3 + X[:, 1] ** 2, 1)).astype(np.float32)
    g, o = both(1, X, y, ntree=4, mtry=3, minndsize=1)
    compare_fit(g, o, 1)
