"""The CPU oracle of the leaf-assignment queries against the reference's own outputs (CPU).

tests/golden/leaves_*.npz were written by tests/golden/make_golden.py (`leaves`) from the
reference module built in oracle/_ref: get_leaf_assignments, get_top_k_similar,
select_outlier_anchors, compute_outlier_scores (greedy and full), compute_outliers,
predict_leaf_assignments and predict_top_k_similar.  Everything is bit for bit except the
'full' outlier scores, whose reference sums float terms in hash-map order (tolerance below).
"""
import os

import numpy as np
import pytest

import oracle
from oracle import leaves as OL

GOLD = os.path.join(os.path.dirname(__file__), "golden")

# name: (task, ntree, mtry, minndsize) as in make_golden.LEAF_CASES
CASES = {"leaves_class": (0, 12, 3, 1), "leaves_regr": (1, 10, 2, 5), "leaves_unsup": (2, 8, 2, 1)}

# 'full' outlier scores: the reference's float32 sum of squares runs in unordered_map order;
# ours is exact and rounded once, so the raw measures differ in the last bits only
FULL_RTOL, FULL_ATOL = 1e-4, 1e-4


def oracle_state(name):
    task, ntree, mtry, nds = CASES[name]
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    X = g["X"]
    n = X.shape[0]
    y = g["y"] if "y" in g else None
    o = oracle.fit(task, X, y, ntree=ntree, mtry=mtry, minndsize=nds,
                   maxnode=oracle.maxnode(2 * n if task == 2 else n, nds), importance=False)
    Xall = oracle.synthetic(X) if task == 2 else X
    lv = OL.leaf_assignments(o, Xall)
    return g, o, lv, o["nin"] == 0


@pytest.fixture(scope="module", params=sorted(CASES))
def state(request):
    return (request.param,) + oracle_state(request.param)


def test_leaf_assignments(state):
    name, g, o, lv, oob = state
    np.testing.assert_array_equal(lv, g["leaves"])


def test_top_k_similar(state):
    name, g, o, lv, oob = state
    for ex in (1, 0):
        for qi, q in enumerate(g["queries"]):
            idx, sim = OL.top_k_similar(lv, oob, int(q), 10, bool(ex))
            m = idx.shape[0]
            np.testing.assert_array_equal(idx, g[f"topk_idx_ex{ex}"][qi, :m])
            np.testing.assert_array_equal(sim, g[f"topk_sim_ex{ex}"][qi, :m])
            assert (g[f"topk_idx_ex{ex}"][qi, m:] == -1).all()


def test_outlier_scores(state):
    name, g, o, lv, oob = state
    task = CASES[name][0]
    labels = g["y"] if task == 0 else None
    greedy = OL.outlier_scores(OL.outlier_raw_greedy(lv, g["anchors_random"], 25), labels)
    np.testing.assert_array_equal(greedy, g["outlier_greedy"])
    full = OL.outlier_scores(OL.outlier_raw_full(lv), labels)
    np.testing.assert_allclose(full, g["outlier_full"], rtol=FULL_RTOL, atol=FULL_ATOL)


def test_predict_outlier_scores(state):
    name, g, o, lv, oob = state
    task = CASES[name][0]
    p = g["X"].shape[1]
    labels = g["y"] if task == 0 else None
    stats = OL.outlier_stats(OL.outlier_raw_greedy(lv, g["anchors_random"], 25), labels)
    nl = OL.predict_leaf_assignments(o, g["Xn"], np.ones(p, np.int32))
    classes = None
    if task == 0:
        classes, _ = oracle.predict(0, o, g["Xn"], int(g["y"].max()) + 1, np.ones(p, np.int32))
    full = OL.predict_outlier_scores(lv, nl, stats, False, 100, classes)
    greedy = OL.predict_outlier_scores(lv, nl, stats, True, 7, classes)
    np.testing.assert_array_equal(full, g["new_outlier_full"])
    np.testing.assert_array_equal(greedy, g["new_outlier_greedy"])


def test_predict_leaves_and_similar(state):
    name, g, o, lv, oob = state
    p = g["X"].shape[1]
    nl = OL.predict_leaf_assignments(o, g["Xn"], np.ones(p, np.int32))
    np.testing.assert_array_equal(nl, g["new_leaves"])
    idx, sim = OL.predict_top_k_similar(lv, nl, 8)
    np.testing.assert_array_equal(idx, g["new_topk_idx"])
    np.testing.assert_array_equal(sim, g["new_topk_sim"])


def test_partial_sort_matches_a_full_sort_on_distinct_keys():
    rng = np.random.default_rng(3)
    a = list(rng.permutation(50))
    OL.partial_sort(a, 10, lambda x, y: x > y)
    assert a[:10] == sorted(a, reverse=True)[:10]
