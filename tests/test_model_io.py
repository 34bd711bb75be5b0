"""The RFX0 model file (RandomForest::save / load, src/rf_random_forest.cpp:5987-6270) on CPU:
reference-written files parse and re-serialise byte for byte, and their trees predict what
the reference predicted (through the oracle's walk)."""
import gzip
import os

import numpy as np
import pytest

import oracle
from rfx_b200 import model_io

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def unpack(name, tmp_path):
    path = tmp_path / f"{name}.rfx"
    with gzip.open(os.path.join(GOLD, f"{name}.rfx.gz"), "rb") as g:
        path.write_bytes(g.read())
    return path


@pytest.mark.parametrize("name", ["predict_class", "predict_regr", "unsup_model"])
def test_reference_file_round_trips(name, tmp_path):
    src = unpack(name, tmp_path)
    m = model_io.read(str(src))
    assert m["ntree"] >= 1 and m["nodestatus"].size == m["ntree"] * m["maxnode"]
    out = tmp_path / "rewritten.rfx"
    model_io.write(str(out), m)
    assert out.read_bytes() == src.read_bytes()


@pytest.mark.parametrize("name", ["predict_class", "predict_regr"])
def test_reference_file_trees_predict_like_the_reference(name, tmp_path):
    m = model_io.read(str(unpack(name, tmp_path)))
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    T = m["ntree"]
    trees = {k: m[k].reshape(T, -1) for k in ("nodestatus", "bestvar", "xbestsplit", "treemap",
                                              "nodeclass", "nodepred")}
    if m["task_type"] == 0:
        cls, proba = oracle.predict(0, trees, g["Xn"], m["nclass"], m["cat"], [0.3, 1.0, 0.6, 0.9])
        assert np.array_equal(m["label_inverse"][cls], g["pred"])
        assert np.array_equal(proba, g["proba"].astype(np.float32))
    else:
        pred = oracle.predict(1, trees, g["Xn"], 1, m["cat"])
        assert np.array_equal(pred.view(np.uint32), g["pred"].astype(np.float32).view(np.uint32))


def test_bad_magic_is_rejected(tmp_path):
    p = tmp_path / "bad.rfx"
    p.write_bytes(b"XXXX" + bytes(16))
    with pytest.raises(RuntimeError, match="bad magic"):
        model_io.read(str(p))
