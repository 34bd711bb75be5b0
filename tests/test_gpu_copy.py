"""The tree arrays a fit returns are the same whichever host copy carried them.

Arrays of more than 4 MB per batch leave the device through the pinned staging buffers (in
32 MB chunks); small ones through a plain copy.  A 500-tree fit on 50,000 rows in one batch
(two chunks per array) must return exactly the arrays of the same fit in 10-tree batches.
"""
import numpy as np
import pytest

from _helpers import synth

pytestmark = pytest.mark.gpu


def test_staged_and_direct_tree_copies_agree():
    import rfx_b200
    X, y = synth("regr", 50000, 6, 12)
    out = []
    for bt in (500, 10):
        m = rfx_b200.RandomForestRegressor(nsample=50000, ntree=500, mtry=2, minndsize=5,
                                           compute_importance=False, batch_trees=bt)
        m.fit(X, y)
        out.append(m.trees_)
    big, small = out
    assert big["treemap"].nbytes > 64 << 20  # two 32 MB chunks at least
    for k in ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodepred", "nnode", "tnodewt"):
        assert np.array_equal(big[k].view(np.uint32) if big[k].dtype == np.float32 else big[k],
                              small[k].view(np.uint32) if small[k].dtype == np.float32 else small[k]), k
