"""predict / predict_proba of new rows on the device (rfx_predict), bit for bit.

* against the reference's own predictions of the golden fixtures (out-of-range categories
  and NaNs included);
* against the oracle's restatement of the reference walk on the device-grown trees at larger
  sizes, classwt-weighted votes included;
* through rfx_load_forest with trees grown elsewhere (the oracle's);
* inputs with nsample rows return the stored OOB results, as the reference does.
"""
import os

import numpy as np
import pytest

import oracle
from _helpers import synth

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", ["predict_class", "predict_regr"])
def test_predict_matches_reference_golden(name):
    import rfx_b200
    g = dict(np.load(os.path.join(GOLD, f"{name}.npz")))
    X, Xn = g["X"], g["Xn"]
    n, p = X.shape
    if name == "predict_class":
        est = rfx_b200.RandomForestClassifier(nsample=n, ntree=5, mdim=p, mtry=3, minndsize=1,
                                              compute_importance=False,
                                              classwt=[0.3, 1.0, 0.6, 0.9])
        est.fit(X, g["y"])
        assert np.array_equal(est.predict(Xn), g["pred"])
        assert np.array_equal(_bits(est.predict_proba(Xn)), _bits(g["proba"]))
    else:
        est = rfx_b200.RandomForestRegressor(nsample=n, ntree=5, mdim=p, mtry=3, minndsize=3,
                                             compute_importance=False)
        est.fit(X, g["y"])
        assert np.array_equal(_bits(est.predict(Xn)), _bits(g["pred"]))


def _with_categorical(X, seed):
    rng = np.random.default_rng(seed)
    c = rng.integers(0, 6, X.shape[0]).astype(np.float32)
    return np.concatenate([X, c[:, None]], axis=1)


def test_predict_classification_vs_oracle():
    import rfx_b200
    X, y = synth("multiclass", 26000, 10, 41)
    X = _with_categorical(X, 41)
    Xt, yt, Xn = X[:6000], y[:6000], X[6000:]
    Xn[:100, -1] = 9.0
    est = rfx_b200.RandomForestClassifier(nsample=6000, ntree=40, mdim=X.shape[1], mtry=4,
                                          minndsize=1, compute_importance=False,
                                          classwt=[0.2, 1.0, 0.5, 0.7])
    est.fit(Xt, yt)
    cls, proba = oracle.predict(0, est.trees_, Xn, est.nclass_, est._cat, est.classwt_)
    assert np.array_equal(est.predict(Xn), est.classes_[cls])
    assert np.array_equal(_bits(est.predict_proba(Xn)), _bits(proba))


def test_predict_regression_vs_oracle():
    import rfx_b200
    X, y = synth("regr", 25000, 12, 42)
    est = rfx_b200.RandomForestRegressor(nsample=5000, ntree=30, mdim=12, mtry=4, minndsize=5,
                                         compute_importance=False)
    est.fit(X[:5000], y[:5000])
    want = oracle.predict(1, est.trees_, X[5000:], 1, np.ones(12, np.int32))
    assert np.array_equal(_bits(est.predict(X[5000:])), _bits(want))


def test_load_forest_with_oracle_trees():
    import rfx_b200
    from rfx_b200 import _abi as A
    X, y = synth("class", 3000, 8, 43)
    M = oracle.maxnode(2000, 1, 0)
    o = oracle.fit(0, X[:2000], y[:2000], ntree=12, mtry=3, minndsize=1, maxnode=M,
                   importance=False)
    cat = np.ones(8, np.int32)
    ctx = rfx_b200.Context(0)
    ctx.load_forest(A.TASK_CLASSIFICATION, o, cat, nclass=o["nclass"])
    cls, proba = ctx.predict(X[2000:], o["nclass"])
    wc, wp = oracle.predict(0, o, X[2000:], o["nclass"], cat)
    assert np.array_equal(cls, wc) and np.array_equal(_bits(proba), _bits(wp))


def test_training_size_input_returns_oob_results():
    import rfx_b200
    X, y = synth("class", 1500, 6, 44)
    est = rfx_b200.RandomForestClassifier(nsample=1500, ntree=10, mdim=6, mtry=2, minndsize=1,
                                          compute_importance=False)
    est.fit(X, y)
    Xother = np.random.default_rng(1).normal(size=X.shape).astype(np.float32)
    assert np.array_equal(est.predict(Xother), est.classes_[est._oob_class])
    assert np.array_equal(est.predict_proba(Xother), est._oob_proba)
