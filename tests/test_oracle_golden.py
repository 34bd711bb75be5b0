"""The CPU oracle against golden vectors produced by the reference itself (CPU only).

tests/golden/*.npz were written by tests/golden/make_golden.py from the reference build in
oracle/_ref.  Everything is compared bit for bit: tree arrays, bootstrap counts, terminal
nodes, OOB counts and vote sums, OOB predictions, importance, proximity sums and the
finishprox'd matrix, quantile bin edges and codes.
"""
import os

import numpy as np
import pytest

import oracle
from _helpers import assert_same

GOLD = os.path.join(os.path.dirname(__file__), "golden")

CASES = {
    "class_prox": (0, dict(ntree=4, mtry=3, minndsize=1, proximity=True)),
    "multiclass_classwt": (0, dict(ntree=3, mtry=2, minndsize=2, classwt=[0.1, 0.4, 0.7, 1.0])),
    "regr": (1, dict(ntree=3, mtry=4, minndsize=5)),
    "regr_bins16_cap": (1, dict(ntree=3, mtry=3, minndsize=2, nbins=16)),
    "unsup_prox": (2, dict(ntree=3, mtry=2, minndsize=1, proximity=True)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_fit(name):
    task, kw = CASES[name]
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    y = g["y"] if "y" in g else None
    o = oracle.fit(task, g["X"], y, maxnode=int(g["maxnode"]), **kw)
    for k in ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass", "nnode", "tnodewt",
              "nin", "nout", "avimp", "sqsd"):
        assert_same(k, o[k], g[k])
    oob = g["nin"] == 0
    if kw.get("proximity"):
        assert_same("nodextr", o["nodextr"], g["nodextr"])
    else:
        assert_same("nodextr(oob)", np.where(oob, o["nodextr"], 0), np.where(oob, g["nodextr"], 0))
    if task == 1:
        assert_same("nodepred", o["nodepred"], g["nodepred"])
        assert_same("oob_pred", o["oob_pred"], g["oob_pred"])
    else:
        assert_same("q", o["q"], g["q"])
    assert np.float32(o["oob_error"]) == np.float32(g["oob_error"])
    if kw.get("proximity"):
        assert_same("prox_pairs", o["prox_pairs"], g["prox_pairs"])
        assert_same("prox", o["prox"], g["prox"])


def test_oracle_bootstrap_matches_reference():
    g = np.load(os.path.join(GOLD, "bootstrap.npz"))
    for t in range(g["nin"].shape[0]):
        assert_same("nin", oracle.bootstrap(900, t), g["nin"][t])
        assert_same("nin_w", oracle.bootstrap(900, t, sample_weights=g["sw"]), g["nin_w"][t])


@pytest.mark.parametrize("nbins,suffix", [(256, ""), (16, "16")])
def test_oracle_binning_matches_reference(nbins, suffix):
    g = np.load(os.path.join(GOLD, "binning.npz"))
    e, nb, kind, xb = oracle.binning(g["X"], g["cat"], nbins)
    assert_same("nb", nb, g["nb" + suffix])
    assert_same("kind", kind, g["kind" + suffix])
    assert_same("xb", xb, g["xb" + suffix])
    for f in range(len(nb)):
        if kind[f] != 2:  # categorical features keep the reference's zeroed edge array
            assert_same(f"edges[{f}]", e[f, : nb[f] + 1], g["edges" + suffix][f, : nb[f] + 1])


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
def test_oracle_matches_reference_on_fresh_case():
    """Direct cross-check on a case the fixtures do not hold (where the reference is built)."""
    from _helpers import synth
    X, y = synth("regr", 900, 9, 21)
    r = oracle.ref_fit(1, X, y, ntree=2, mtry=3, minndsize=3)
    o = oracle.fit(1, X, y, ntree=2, mtry=3, minndsize=3, maxnode=r["maxnode"])
    for k in ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodepred", "nin", "avimp"):
        assert_same(k, o[k], r[k])


@pytest.mark.parametrize("name", ["predict_class", "predict_regr"])
def test_oracle_predict_matches_reference(name):
    """orc_predict on the oracle's trees equals the reference's predict()/predict_proba() of
    new rows, including out-of-range categories and NaNs."""
    g = dict(np.load(os.path.join(GOLD, f"{name}.npz"), allow_pickle=False))
    task = 0 if name == "predict_class" else 1
    X, y, Xn, cat = g["X"], g.get("y"), g["Xn"], g["cat"]
    M = int(g["maxnode"])
    kw = dict(ntree=5, mtry=3, minndsize=1 if task == 0 else 3, maxnode=M, cat=cat,
              importance=False)
    if task == 0:
        kw["classwt"] = [0.3, 1.0, 0.6, 0.9]
    o = oracle.fit(task, X, y, **kw)
    if task == 0:
        labels = np.unique(y)
        cls, proba = oracle.predict(0, o, Xn, o["nclass"], cat, kw["classwt"])
        assert np.array_equal(labels[cls], g["pred"])
        assert np.array_equal(proba.view(np.uint32), g["proba"].astype(np.float32).view(np.uint32))
    else:
        pred = oracle.predict(1, o, Xn, 1, cat)
        assert np.array_equal(pred.view(np.uint32), g["pred"].astype(np.float32).view(np.uint32))
