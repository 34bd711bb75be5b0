"""Shared helpers for the parity tests: run the device path through the C ABI and the
oracle on the same inputs, and compare bit for bit."""
from __future__ import annotations

import numpy as np

import oracle
import rfx_b200
from rfx_b200 import _abi as A


def synth(kind: str, n: int, p: int, seed: int):
    rng = np.random.default_rng(seed)
    if kind == "class":
        X = rng.normal(size=(n, p)).astype(np.float32)
        w = rng.normal(size=p)
        y = (rng.random(n) < 1 / (1 + np.exp(-X @ w))).astype(np.int32)
        return X, y
    if kind == "multiclass":
        k = 4
        mu = rng.normal(scale=1.5, size=(k, p))
        y = rng.integers(0, k, size=n).astype(np.int32)
        X = (mu[y] + rng.normal(size=(n, p))).astype(np.float32)
        return X, y
    if kind == "regr":
        X = rng.uniform(-1, 1, size=(n, p)).astype(np.float32)
        y = np.sin(3 * X[:, : min(p, 10)]).sum(1)
        if p > 11:
            y = y + 0.5 * X[:, 10] * X[:, 11]
        y = (y + rng.normal(scale=0.1, size=n)).astype(np.float32)
        return X, y
    if kind == "gmm":
        k = 5
        mu = rng.normal(scale=4.0, size=(k, p))
        var = rng.uniform(0.5, 2.0, size=(k, p))
        z = rng.integers(0, k, size=n)
        X = (mu[z] + rng.normal(size=(n, p)) * np.sqrt(var[z])).astype(np.float32)
        return X, None
    raise ValueError(kind)


def gpu_fit(task, X, y=None, *, ntree, mtry, minndsize, maxnode, iseed=12345, nbins=256,
            sample_weights=None, cat=None, classwt=None, importance=True, proximity=False,
            batch_trees=0, maxcat=10, ctx=None, tree_chunks=None, prox_rows=0, fetch_prox=True):
    """Device fit through the C ABI; returns a dict shaped like oracle.fit's."""
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    N = 2 * n if task == 2 else n
    ncl = len(np.unique(y)) if task == 0 else (2 if task == 2 else 1)
    prm = A.FitParams(task, n, p, mtry, minndsize, maxnode, iseed, 12345, nbins, maxcat,
                      int(importance), int(proximity), prox_rows, batch_trees, 0)
    ycls = np.ascontiguousarray(y, np.int32) if task == 0 else None
    yreg = np.ascontiguousarray(y, np.float32) if task == 1 else None
    sw = None if sample_weights is None else np.ascontiguousarray(sample_weights, np.float32)
    c = None if cat is None else np.ascontiguousarray(cat, np.int32)
    cw = None if classwt is None else np.ascontiguousarray(classwt, np.float32)
    inp = A.Inputs(A.ptr(X, A._pf), A.ptr(ycls, A._pi), A.ptr(yreg, A._pf), A.ptr(sw, A._pf),
                   A.ptr(c, A._pi), A.ptr(cw, A._pf))
    M, T = maxnode, ntree
    r = {
        "nodestatus": np.zeros((T, M), np.int32), "bestvar": np.zeros((T, M), np.int32),
        "xbestsplit": np.zeros((T, M), np.float32), "treemap": np.zeros((T, 2 * M), np.int32),
        "nodeclass": np.zeros((T, M), np.int32), "nnode": np.zeros(T, np.int32),
        "nodepred": np.zeros((T, M), np.float32), "tnodewt": np.zeros((T, M), np.float32),
        "nin": np.zeros((T, N), np.int32), "oob_leaf": np.zeros((T, N), np.int32),
        "tree_rr": np.zeros((T, p), np.float32), "tree_used": np.zeros((T, p), np.uint8),
    }
    keys = ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass", "nnode", "nodepred",
            "tnodewt", "nin", "oob_leaf", "tree_rr", "tree_used")
    types = (A._pi, A._pi, A._pf, A._pi, A._pi, A._pi, A._pf, A._pf, A._pi, A._pi, A._pf, A._pu8)
    ctx = ctx or rfx_b200.Context(0)
    ctx.load(prm, inp)
    chunks = tree_chunks or [T]
    t0 = 0
    for k in chunks:
        # row slices of C-ordered arrays are contiguous views: the ABI writes in place
        tr = A.Trees(*[A.ptr(r[key][t0:t0 + k], t) for key, t in zip(keys, types)])
        ctx.grow(t0, k, tr)
        t0 += k
    acc = {"nout": np.zeros(N, np.int32), "votes": np.zeros((N, ncl), np.int32),
           "q": np.zeros((N, ncl), np.float32), "oob_sum": np.zeros(N, np.float32),
           "avimp": np.zeros(p, np.float32), "sqsd": np.zeros(p, np.float32),
           "labels": np.zeros(N, np.int32)}
    ac = A.Accum(0, 0, *[A.ptr(acc[k], t) for k, t in (
        ("nout", A._pi), ("votes", A._pi), ("q", A._pf), ("oob_sum", A._pf), ("avimp", A._pf),
        ("sqsd", A._pf), ("labels", A._pi))])
    if ncl == 1:
        ac.votes = ac.q = ac.labels = None
    ctx.results(ac)
    r.update(acc)
    if proximity and fetch_prox:
        dev, length = ctx.prox_buffer()
        up = np.empty(length, np.int32)
        ctx.copy_to_host(up, dev)
        r["prox_upper"] = up
        r["prox"] = np.empty((N, N), np.float32)
        ctx.prox_dense(0, N, r["prox"])
    r["ctx"] = ctx
    return r


def upper_from_pairs(P: np.ndarray) -> np.ndarray:
    C = P + P.T
    iu = np.triu_indices(P.shape[0], 1)
    return C[iu].astype(np.int32)


def bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else (a.view(np.uint64) if a.dtype == np.float64 else a)


def assert_same(name, a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, f"{name}: shape {a.shape} vs {b.shape}"
    bad = np.argwhere(bits(a) != bits(b))
    assert len(bad) == 0, f"{name}: {len(bad)} mismatches, first {bad[:5].tolist()} " \
                          f"got {a[tuple(bad[0])]} want {b[tuple(bad[0])]}"


def compare_fit(g, o, task, proximity=False, importance=True):
    for k in ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass", "nnode", "nodepred", "tnodewt"):
        assert_same(k, g[k], o[k])
    assert_same("nin", g["nin"], o["nin"])
    oob = o["nin"] == 0
    assert_same("oob_leaf", np.where(oob, g["oob_leaf"], -1), np.where(oob, o["nodextr"], -1))
    assert_same("nout", g["nout"], o["nout"])
    if task == 1:
        assert_same("oob_sum", g["oob_sum"], o["oob_sum"])
    else:
        assert_same("votes", g["votes"], o["votes"])
        assert_same("q", g["q"], o["q"])
    if importance:
        assert_same("tree_rr", g["tree_rr"], o["tree_rr"])
        assert_same("avimp", g["avimp"], o["avimp"])
        assert_same("sqsd", g["sqsd"], o["sqsd"])
    if proximity:
        assert_same("prox_upper", g["prox_upper"], upper_from_pairs(o["prox_pairs"]))
        assert_same("prox", g["prox"], o["prox"].astype(np.float32))


def inbag_leaves(g, X, t):
    """Terminal node of every row of X in tree t of a device fit (raw x <= split, the walk
    the grower's partition makes; every feature quantitative)."""
    st, bv, xb, tm = g["nodestatus"][t], g["bestvar"][t], g["xbestsplit"][t], g["treemap"][t]
    node = np.zeros(X.shape[0], np.int64)
    rows = np.arange(X.shape[0])
    for _ in range(100000):
        live = st[node] == 1
        if not live.any():
            return node
        r = rows[live]
        nd = node[live]
        left = X[r, bv[nd]] <= xb[nd]
        node[r] = np.where(left, tm[2 * nd], tm[2 * nd + 1])
    raise AssertionError("tree walk did not terminate")


def expected_counts(g, X, R, rows):
    """C[i, j] = P_ij + P_ji for the given rows i (all j < R): the reference's dense proximity
    (src/rf_proximity.cpp:99-230): OOB row i in leaf k meets every distinct in-bag row of k."""
    C = np.zeros((len(rows), R), np.int32)
    for t in range(g["nin"].shape[0]):
        leaf = inbag_leaves(g, X[:R], t)
        oob = g["nin"][t, :R] == 0
        assert np.array_equal(leaf[oob], g["oob_leaf"][t, :R][oob])
        eq = leaf[rows][:, None] == leaf[None, :]
        C += (eq & (oob[rows][:, None] & ~oob[None, :])).astype(np.int32)
        C += (eq & (~oob[rows][:, None] & oob[None, :])).astype(np.int32)
    return C


def device_upper_rows(ctx, R, rows):
    """C[i, i+1:R] of the given rows from the device's packed upper triangle."""
    dev, length = ctx.prox_buffer()
    assert length == R * (R - 1) // 2
    out = {}
    for i in rows:
        off = i * (2 * R - i - 1) // 2
        seg = np.empty(R - i - 1, np.int32)
        if len(seg):
            ctx.copy_to_host(seg, int(dev) + 4 * int(off))
        out[int(i)] = seg
    return out


def finish_rows(C, rows, nout):
    """finishprox (src/rf_finishprox.cpp:12-74, the oracle's double operations) for the given
    rows of C = P + P^T, as float32."""
    inv = np.where(nout > 0, 1.0 / np.maximum(nout, 1).astype(np.float64), 1.0)
    a = C.astype(np.float64) / 2.0
    si = a * inv[rows][:, None]
    sj = a * inv[None, :C.shape[1]]
    S = 0.5 * (si + sj)
    S[np.arange(len(rows)), rows] = 1.0
    return S.astype(np.float32)
