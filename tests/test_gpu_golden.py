"""The device path against the reference's own golden vectors (tests/golden/), bit for bit."""
import os

import numpy as np
import pytest

from _helpers import assert_same, gpu_fit, upper_from_pairs
from test_oracle_golden import CASES, GOLD

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(CASES))
def test_device_matches_reference_golden(name):
    task, kw = CASES[name]
    g = np.load(os.path.join(GOLD, f"{name}.npz"))
    y = g["y"] if "y" in g else None
    d = gpu_fit(task, g["X"], y, maxnode=int(g["maxnode"]), **kw)
    for k in ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass", "nnode", "tnodewt",
              "nin", "nout", "avimp", "sqsd"):
        assert_same(k, d[k], g[k])
    oob = g["nin"] == 0
    assert_same("oob_leaf", np.where(oob, d["oob_leaf"], -1), np.where(oob, g["nodextr"], -1))
    if task == 1:
        assert_same("nodepred", d["nodepred"], g["nodepred"])
        nout = d["nout"]
        pred = np.where(nout > 0, d["oob_sum"] / np.maximum(nout, 1).astype(np.float32), d["oob_sum"])
        assert_same("oob_pred", pred.astype(np.float32), g["oob_pred"])
    else:
        assert_same("q", d["q"], g["q"])
    if kw.get("proximity"):
        assert_same("prox_upper", d["prox_upper"], upper_from_pairs(g["prox_pairs"]))
        assert_same("prox", d["prox"], g["prox"].astype(np.float32))
