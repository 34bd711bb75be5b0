"""Leaf assignments and the queries on them, on the device (csrc/rfx_leaves.cu).

* against the reference's own outputs (tests/golden/leaves_*.npz, written from the reference
  module by make_golden.py): get_leaf_assignments, get_top_k_similar (both exclude_self
  settings, the reference's tie order), select_outlier_anchors (random and diverse),
  compute_outlier_scores (greedy bit for bit; full within the tolerance of
  test_oracle_leaves), compute_outliers, predict_outlier_scores, predict_leaf_assignments,
  predict_top_k_similar;
* against the oracle's restatement on the device-grown trees at a larger size.
"""
import os

import numpy as np
import pytest

import oracle
from oracle import leaves as OL
from _helpers import synth
from test_oracle_leaves import CASES, FULL_ATOL, FULL_RTOL

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _fit(task, X, y, ntree, mtry, nds):
    import rfx_b200
    n = X.shape[0]
    kw = dict(nsample=n, ntree=ntree, mtry=mtry, minndsize=nds, compute_importance=False,
              compute_proximity=False, compute_leaf_assignments=True)
    if task == 0:
        m = rfx_b200.RandomForestClassifier(**kw)
        m.fit(X, y)
    elif task == 1:
        m = rfx_b200.RandomForestRegressor(**kw)
        m.fit(X, y)
    else:
        m = rfx_b200.RandomForestUnsupervised(**kw)
        m.fit(X)
    return m


@pytest.mark.parametrize("name", sorted(CASES))
def test_leaf_queries_match_reference_golden(name):
    task, ntree, mtry, nds = CASES[name]
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    y = g["y"] if "y" in g else None
    m = _fit(task, g["X"], y, ntree, mtry, nds)
    np.testing.assert_array_equal(m.get_leaf_assignments(), g["leaves"])
    for ex in (1, 0):
        for qi, q in enumerate(g["queries"]):
            ref_idx = g[f"topk_idx_ex{ex}"][qi]
            if (ref_idx == -1).all():
                with pytest.raises(RuntimeError):
                    m.get_top_k_similar(int(q), 10, bool(ex))
                continue
            idx, sim = m.get_top_k_similar(int(q), 10, bool(ex))
            k = idx.shape[0]
            np.testing.assert_array_equal(idx, ref_idx[:k])
            np.testing.assert_array_equal(sim, g[f"topk_sim_ex{ex}"][qi, :k])
            assert (ref_idx[k:] == -1).all()
    # the reference's call sequence: anchors random 25, diverse 12, then greedy with 25
    # anchors (re-selected at random because the stored ones number 12), then full
    np.testing.assert_array_equal(m.select_outlier_anchors(25, "random"), g["anchors_random"])
    np.testing.assert_array_equal(m.select_outlier_anchors(12, "diverse"), g["anchors_diverse"])
    np.testing.assert_array_equal(m.compute_outlier_scores("greedy", 25), g["outlier_greedy"])
    full = m.compute_outlier_scores("full", 100)
    np.testing.assert_allclose(full, g["outlier_full"], rtol=FULL_RTOL, atol=FULL_ATOL)
    oi, osc = m.compute_outliers(7, "full", 100)
    # ranking of our scores with the reference's sort; same rows where no near-ties separate them
    ref = g["outliers_score"]
    if np.all(np.diff(ref) < -1e-3):
        np.testing.assert_array_equal(oi, g["outliers_idx"])
    np.testing.assert_allclose(osc, ref, rtol=FULL_RTOL, atol=FULL_ATOL)
    # new rows, normalised by the greedy training statistics (exact on both sides)
    m.compute_outlier_scores("greedy", 25)
    np.testing.assert_array_equal(m.predict_outlier_scores(g["Xn"], "full", 100), g["new_outlier_full"])
    np.testing.assert_array_equal(m.predict_outlier_scores(g["Xn"], "greedy", 7), g["new_outlier_greedy"])
    np.testing.assert_array_equal(m.predict_leaf_assignments(g["Xn"]), g["new_leaves"])
    ti, ts = m.predict_top_k_similar(g["Xn"], 8)
    np.testing.assert_array_equal(ti, g["new_topk_idx"])
    np.testing.assert_array_equal(ts, g["new_topk_sim"])


def test_leaf_queries_match_oracle_larger():
    """A 4000-row regression forest of 24 trees: every query against the oracle's
    restatement over the same (device-grown) trees."""
    X, y = synth("regr", 4300, 8, 77)
    Xn = X[4000:]
    X, y = X[:4000], y[:4000]
    m = _fit(1, X, y, 24, 3, 3)
    tr = m.trees_
    lv = OL.leaf_assignments(tr, X)
    np.testing.assert_array_equal(m.get_leaf_assignments(), lv)
    oob = oracle.fit(1, X, y, ntree=24, mtry=3, minndsize=3,
                     maxnode=oracle.maxnode(4000, 3), importance=False)["nin"] == 0
    for q in (0, 5, 1999, 3999):
        idx, sim = m.get_top_k_similar(q, 25, True)
        oi, os_ = OL.top_k_similar(lv, oob, q, 25, True)
        np.testing.assert_array_equal(idx, oi)
        np.testing.assert_array_equal(sim, os_)
        assert m.compute_proximity_from_leaves(q, int(oi[0])) == OL.leaf_proximity(lv, oob, q, int(oi[0]))
    anchors = m.select_outlier_anchors(40, "random")
    np.testing.assert_array_equal(m.compute_outlier_scores("greedy", 40),
                                  OL.outlier_scores(OL.outlier_raw_greedy(lv, anchors, 40)))
    np.testing.assert_allclose(m.compute_outlier_scores("full"),
                               OL.outlier_scores(OL.outlier_raw_full(lv)), rtol=1e-6, atol=1e-6)
    nl = OL.predict_leaf_assignments(tr, Xn, np.ones(8, np.int32))
    np.testing.assert_array_equal(m.predict_leaf_assignments(Xn), nl)
    st = OL.outlier_stats(OL.outlier_raw_full(lv))  # the last training scores were 'full'
    for mode, na in (("full", 100), ("greedy", 9)):
        np.testing.assert_allclose(m.predict_outlier_scores(Xn[:30], mode, na),
                                   OL.predict_outlier_scores(lv, nl[:30], st, mode == "greedy", na),
                                   rtol=1e-6, atol=1e-6)
    ti, ts = m.predict_top_k_similar(Xn[:40], 12)
    oi, os_ = OL.predict_top_k_similar(lv, nl[:40], 12)
    np.testing.assert_array_equal(ti, oi)
    np.testing.assert_array_equal(ts, os_)


def test_leaf_queries_need_compute_leaf_assignments():
    X, y = synth("regr", 300, 4, 5)
    import rfx_b200
    m = rfx_b200.RandomForestRegressor(nsample=300, ntree=3, mtry=2, compute_importance=False)
    m.fit(X, y)
    with pytest.raises(RuntimeError):
        m.get_leaf_assignments()
    with pytest.raises(RuntimeError):
        m.get_top_k_similar(0)
