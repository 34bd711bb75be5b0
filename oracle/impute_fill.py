"""CPU restatement of one fill round of rfx_impute_proximity (python/rfx_impute.py:730-771)
with every aggregation: 'mean' / 'weighted_mean' (proximity-weighted mean, categorical:
proximity-weighted mode) and 'median' (median, categorical: most frequent value), over all
observed rows with positive proximity or, with top_k, over the top_k of them.

Test infrastructure: only tests/ and bench.py's CPU legs use it.

The reference selects the top_k with np.argsort (the default kind), whose order among equal
proximities is implementation-defined; this restatement (and the device) use the stable
order: ascending proximity, ties by ascending row, the last top_k kept in that order.
"""
import numpy as np


def fill(prox, X, missing, cat, cells, top_k=None, aggregation="mean", sort_kind="stable"):
    """New float32 value of each (row, column) cell, NaN where the reference keeps the old
    one (no other observed row with positive proximity).  prox: row-indexable finished
    proximity (prox[i] a float32 row of length n); X: current float32 values.  sort_kind None
    is the reference's own np.argsort call (numpy's default sort)."""
    out = np.full(len(cells), np.nan, np.float32)
    for c, (i, j) in enumerate(cells):
        s = np.array(prox[i, :], np.float32, copy=True)  # rfx_impute.py:736-740
        s[i] = 0
        observed = ~missing[:, j]
        s[~observed] = 0
        obs = np.where(observed & (s > 0))[0]
        if len(obs) == 0:
            continue
        if top_k is not None and len(obs) > top_k:  # rfx_impute.py:744-748
            sel = obs[np.argsort(s[obs], kind=sort_kind)[-top_k:]]
        else:
            sel = obs
        vals = X[sel, j]
        w = s[sel]
        if cat[j]:  # rfx_impute.py:753-759
            u = np.unique(vals)
            if aggregation == "median":
                counts = np.array([(vals == v).sum() for v in u])
            else:
                counts = np.array([w[vals == v].sum() for v in u])
            out[c] = u[np.argmax(counts)]
        elif aggregation == "median":  # rfx_impute.py:761-762
            # a zero median as +0 (np.median returns whichever signed zero its partition
            # places in the middle)
            out[c] = np.float32(np.median(vals)) + np.float32(0.0)
        elif aggregation in ("mean", "weighted_mean"):  # rfx_impute.py:763-765
            w = w / w.sum()
            out[c] = np.float32(float(np.sum(w * vals)))
        else:
            raise ValueError(f"Unknown aggregation: {aggregation}")
    return out
