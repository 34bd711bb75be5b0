"""Models fitted on the device save as the reference's RFX0 file byte for byte (same data
and parameters as the reference-written fixtures), and reference files load and predict."""
import gzip
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def ref_bytes(name):
    with gzip.open(os.path.join(GOLD, f"{name}.rfx.gz"), "rb") as g:
        return g.read()


def test_classifier_save_matches_reference_file(tmp_path):
    import rfx_b200
    g = np.load(os.path.join(GOLD, "predict_class.npz"))
    n, p = g["X"].shape
    est = rfx_b200.RandomForestClassifier(nsample=n, ntree=5, mtry=3, minndsize=1,
                                          compute_importance=False, compute_proximity=False,
                                          classwt=[0.3, 1.0, 0.6, 0.9])
    est.fit(g["X"], g["y"])
    est.save(tmp_path / "m.rfx")
    assert (tmp_path / "m.rfx").read_bytes() == ref_bytes("predict_class")


def test_regressor_save_matches_reference_file(tmp_path):
    import rfx_b200
    g = np.load(os.path.join(GOLD, "predict_regr.npz"))
    n, p = g["X"].shape
    est = rfx_b200.RandomForestRegressor(nsample=n, ntree=5, mtry=3, minndsize=3,
                                         compute_importance=False)
    est.fit(g["X"], g["y"])
    est.save(tmp_path / "m.rfx")
    assert (tmp_path / "m.rfx").read_bytes() == ref_bytes("predict_regr")


def test_unsupervised_save_matches_reference_file(tmp_path):
    import rfx_b200
    X = np.load(os.path.join(GOLD, "unsup_model.npz"))["X"]
    est = rfx_b200.RandomForestUnsupervised(nsample=300, ntree=2, mtry=2, minndsize=1)
    est.fit(X)
    est.save(tmp_path / "m.rfx")
    assert (tmp_path / "m.rfx").read_bytes() == ref_bytes("unsup_model")


@pytest.mark.parametrize("name", ["predict_class", "predict_regr"])
def test_loaded_reference_model_predicts(name, tmp_path):
    """A loaded model predicts like the reference's LoadedModel: the file carries no classwt,
    so votes count 1 each, and inputs with nsample rows give class 0 / uniform
    probabilities (no stored OOB results)."""
    import oracle
    import rfx_b200
    from rfx_b200 import model_io
    path = tmp_path / "m.rfx"
    path.write_bytes(ref_bytes(name))
    model = rfx_b200.load(str(path))
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    if name == "predict_class":
        m = model_io.read(str(path))
        T = m["ntree"]
        trees = {k: m[k].reshape(T, -1) for k in ("nodestatus", "bestvar", "xbestsplit",
                                                  "treemap", "nodeclass", "nodepred")}
        cls, proba = oracle.predict(0, trees, g["Xn"], m["nclass"], m["cat"], None)
        assert np.array_equal(model.predict(g["Xn"]), m["label_inverse"][cls])
        assert np.array_equal(model.predict_proba(g["Xn"]).view(np.uint32), proba.view(np.uint32))
        assert not model.predict(g["X"]).any()
        assert np.all(model.predict_proba(g["X"]) == np.float32(0.25))
    else:
        assert np.array_equal(model.predict(g["Xn"]).view(np.uint32),
                              g["pred"].astype(np.float32).view(np.uint32))
