"""Progress callback between tree batches (the reference's progress_callback_(itree + 1,
ntree), src/rf_random_forest.cpp:600-601): counts per batch, cancellation, and the
estimator's tqdm bar."""
import numpy as np
import pytest

import rfx_b200
from rfx_b200 import _abi as A
from _helpers import gpu_fit, synth

pytestmark = pytest.mark.gpu


def test_progress_called_per_batch_and_cancels():
    X, y = synth("class", 800, 6, 3)
    ctx = rfx_b200.Context(0)
    seen = []
    ctx.set_progress(lambda done, total: seen.append((done, total)) and False)
    gpu_fit(0, X, y, ntree=10, mtry=2, minndsize=1, maxnode=1601, batch_trees=4, ctx=ctx)
    assert seen == [(4, 10), (8, 10), (10, 10)]
    ctx.set_progress(lambda done, total: done >= 4)  # stop after the first batch
    with pytest.raises(A.RfxError) as e:
        gpu_fit(0, X, y, ntree=10, mtry=2, minndsize=1, maxnode=1601, batch_trees=4, ctx=ctx)
    assert e.value.code == -7
    ctx.set_progress(None)
    g = gpu_fit(0, X, y, ntree=10, mtry=2, minndsize=1, maxnode=1601, batch_trees=4, ctx=ctx)
    assert g["nnode"].min() > 1


def test_estimator_progress_bar(capsys):
    X, y = synth("regr", 600, 5, 4)
    est = rfx_b200.RandomForestRegressor(nsample=600, ntree=6, mtry=2, minndsize=3,
                                         show_progress=True, progress_desc="Training",
                                         batch_trees=2)
    est.fit(X, y)
    err = capsys.readouterr().err
    assert "Training" in err
    quiet = rfx_b200.RandomForestRegressor(nsample=600, ntree=6, mtry=2, minndsize=3,
                                           show_progress=False, batch_trees=2)
    quiet.fit(X, y)
    assert np.array_equal(quiet.acc_["oob_sum"], est.acc_["oob_sum"])
