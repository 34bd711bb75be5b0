"""Generate the golden fixtures of tests/golden/ from the reference itself.

The reference's CPU implementation is compiled from its own sources into oracle/_ref
(`make -C oracle ref`); oracle/ref_harness.cpp drives it and dumps the per-tree arrays
that its Python API does not expose.  The reference has no golden vectors of its own, so
these fixtures are the pin of the CPU oracle (tests/test_oracle_golden.py) and, through
it, of the device path.

    python tests/golden/make_golden.py        # rewrites tests/golden/*.npz
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "rfx-fuse_b200"))

import oracle  # noqa: E402
from _helpers import synth  # noqa: E402

KEYS = ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass", "nnode", "nodepred",
        "tnodewt", "nin", "nodextr", "nout", "q", "oob_pred", "avimp", "sqsd", "oob_error")


def binning_data():
    rng = np.random.default_rng(99)
    n = 700
    X = np.empty((n, 7), np.float32)
    X[:, 0] = rng.normal(size=n)
    X[:, 1] = np.round(rng.normal(size=n), 1)          # heavy ties
    X[:, 2] = rng.integers(0, 2, n)                    # binary 0/1
    X[:, 3] = rng.integers(0, 5, n)                    # categorical (cat=5)
    X[:, 4] = 2.5                                      # constant
    X[:, 5] = rng.integers(0, 40, n) * 0.25            # 40 distinct values
    X[:, 6] = rng.exponential(size=n) * 1e-3           # tiny spread
    cat = np.array([1, 1, 1, 5, 1, 1, 1], np.int32)
    return X, cat


CASES = {
    # name: (task, data kind, n, p, seed, fit kwargs)
    "class_prox": (0, "class", 600, 8, 1, dict(ntree=4, mtry=3, minndsize=1, proximity=True)),
    "multiclass_classwt": (0, "multiclass", 800, 6, 2,
                           dict(ntree=3, mtry=2, minndsize=2, classwt=[0.1, 0.4, 0.7, 1.0])),
    "regr": (1, "regr", 1500, 12, 3, dict(ntree=3, mtry=4, minndsize=5)),
    "regr_bins16_cap": (1, "regr", 1200, 8, 4, dict(ntree=3, mtry=3, minndsize=2, nbins=16, maxnode=151)),
    "unsup_prox": (2, "gmm", 300, 6, 5, dict(ntree=3, mtry=2, minndsize=1, proximity=True)),
}


def save_gz(model, path):
    """model.save() (RFX0) gzip-compressed: the tree arrays are mostly zeros."""
    import gzip
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        raw = os.path.join(d, "m.rfx")
        model.save(raw)
        with open(raw, "rb") as f, gzip.GzipFile(path, "wb", mtime=0) as g:
            g.write(f.read())


def predict_data(kind, n, p, seed, n_new):
    """Training data plus new rows for predict(): column p is a 5-level categorical; the new
    rows carry out-of-range categories and NaNs (the reference's edge branches)."""
    X, y = synth(kind, n + n_new, p, seed)
    rng = np.random.default_rng(seed + 100)
    c = rng.integers(0, 5, n + n_new).astype(np.float32)
    X = np.concatenate([X, c[:, None]], axis=1)
    if y is not None and kind != "regr":
        y = np.where(c == 3, (y + 1) % (y.max() + 1), y).astype(np.int32)  # the column matters
    Xn = X[n:].copy()
    Xn[:20, p] = 7.0        # category out of range -> class 0 / root value
    Xn[20:30, p] = -1.0
    Xn[30:40, p] = np.nan
    Xn[40:50, 0] = np.nan   # continuous NaN: goes right
    return X[:n], (y[:n] if y is not None else None), Xn


PREDICT_CASES = {
    "predict_class": (0, "multiclass", 900, 6, 31, dict(ntree=5, mtry=3, minndsize=1,
                                                         classwt=[0.3, 1.0, 0.6, 0.9])),
    "predict_regr": (1, "regr", 900, 6, 32, dict(ntree=5, mtry=3, minndsize=3)),
}


def predict_golden():
    """Reference predictions of new rows (python/randomforest_py.cpp:1860-1883)."""
    import rfx_b200.forest as F
    R = oracle.ref_module()
    out = {}
    for name, (task, kind, n, p, seed, kw) in PREDICT_CASES.items():
        X, y, Xn = predict_data(kind, n, p, seed, 300)
        cat = F.feature_kinds(task, X, 10, None)
        common = dict(nsample=n, ntree=kw["ntree"], mtry=kw["mtry"], minndsize=kw["minndsize"],
                      compute_importance=False, compute_proximity=False, show_progress=False)
        if task == 0:
            m = R.RandomForestClassifier(classwt=kw["classwt"], **common)
            m.fit(X, y)
            d = {"pred": np.asarray(m.predict(Xn)), "proba": np.asarray(m.predict_proba(Xn))}
        else:
            m = R.RandomForestRegressor(**common)
            m.fit(X, y)
            d = {"pred": np.asarray(m.predict(Xn))}
        save_gz(m, os.path.join(HERE, f"{name}.rfx.gz"))  # the reference's RFX0 model file
        d.update(X=X, y=y, Xn=Xn, cat=cat, maxnode=np.int32(oracle.maxnode(n, kw["minndsize"], 0)))
        out[name] = d
    return out


def impute_data(n=400, seed=61):
    """Continuous correlated columns, two small categorical columns, 15% cells missing."""
    rng = np.random.default_rng(seed)
    C = 0.4 * np.ones((5, 5)) + 0.6 * np.eye(5)
    Xc = rng.multivariate_normal(np.zeros(5), C, size=n).astype(np.float32)
    c1 = rng.integers(0, 4, n).astype(np.float32)
    c2 = (Xc[:, 0] > 0).astype(np.float32) + rng.integers(0, 2, n)
    X = np.concatenate([Xc, c1[:, None], c2[:, None]], axis=1)
    X[rng.random(X.shape) < 0.15] = np.nan
    return X


def impute_golden(aggregation="mean"):
    """The reference's rfx_impute_proximity (python/rfx_impute.py:596-793) on impute_data()."""
    sys.path.insert(0, oracle.ref_dir())
    tree = oracle.reference_tree()
    if tree is None:
        raise SystemExit("set RFX_REFERENCE to the reference source tree")
    sys.path.insert(0, os.path.join(tree, "python"))
    import importlib
    ri = importlib.import_module("rfx_impute")
    X = impute_data()
    Xo, info = ri.rfx_impute_proximity(X.copy(), ntree=25, n_iterations=3, use_gpu=False,
                                       iseed=42, minndsize=1, aggregation=aggregation)
    return {"X": X, "X_imputed": np.asarray(Xo, np.float32),
            "n_iterations": np.int32(info["n_iterations"])}


LEAF_CASES = {
    # name: (task, data kind, n, p, seed, ntree, mtry, minndsize)
    "leaves_class": (0, "multiclass", 500, 6, 41, 12, 3, 1),
    "leaves_regr": (1, "regr", 450, 5, 42, 10, 2, 5),
    "leaves_unsup": (2, "gmm", 200, 4, 43, 8, 2, 1),
}


def leaves_golden():
    """Leaf assignments and the queries on them (include/rf_random_forest.hpp:296-365) from
    the reference module: top-k similar rows, outlier scores (full and greedy), anchors,
    new-row leaves and top-k similar."""
    R = oracle.ref_module()
    out = {}
    for name, (task, kind, n, p, seed, ntree, mtry, nds) in LEAF_CASES.items():
        X, y = synth(kind, n + 60, p, seed)
        Xn = X[n:].copy()
        X = X[:n]
        common = dict(ntree=ntree, mtry=mtry, minndsize=nds, compute_importance=False,
                      compute_proximity=False, show_progress=False, compute_leaf_assignments=True)
        if task == 0:
            m = R.RandomForestClassifier(nsample=n, **common)
            m.fit(X, y[:n])
        elif task == 1:
            m = R.RandomForestRegressor(nsample=n, **common)
            m.fit(X, y[:n])
        else:
            m = R.RandomForestUnsupervised(nsample=n, **common)
            m.fit(X)
        d = {"X": X, "Xn": Xn, "leaves": np.asarray(m.get_leaf_assignments())}
        if y is not None:
            d["y"] = np.asarray(y[:n])
        N = d["leaves"].shape[1]
        queries = np.array([0, 1, 7, N // 2, N - 1], np.int32)
        for ex in (1, 0):
            idx, sim = [], []
            for q in queries:
                try:
                    a, b = m.get_top_k_similar(int(q), 10, bool(ex))
                except RuntimeError:
                    a, b = np.zeros(0, np.int32), np.zeros(0, np.float32)
                a = np.full(10, -1, np.int32) if len(a) == 0 else np.pad(np.asarray(a, np.int32), (0, 10 - len(a)), constant_values=-1)
                b = np.pad(np.asarray(b, np.float32), (0, 10 - len(b)), constant_values=np.nan) if len(b) else np.full(10, np.nan, np.float32)
                idx.append(a)
                sim.append(b)
            d[f"topk_idx_ex{ex}"] = np.stack(idx)
            d[f"topk_sim_ex{ex}"] = np.stack(sim)
        d["queries"] = queries
        d["anchors_random"] = np.asarray(m.select_outlier_anchors(25, "random"))
        d["anchors_diverse"] = np.asarray(m.select_outlier_anchors(12, "diverse"))
        d["outlier_greedy"] = np.asarray(m.compute_outlier_scores("greedy", 25))
        d["outlier_full"] = np.asarray(m.compute_outlier_scores("full", 100))
        oi, os_ = m.compute_outliers(7, "full", 100)
        d["outliers_idx"], d["outliers_score"] = np.asarray(oi), np.asarray(os_)
        # new-row outlier scores, normalised by the (exact) greedy training statistics
        m.compute_outlier_scores("greedy", 25)
        d["new_outlier_full"] = np.asarray(m.predict_outlier_scores(Xn, "full", 100))
        d["new_outlier_greedy"] = np.asarray(m.predict_outlier_scores(Xn, "greedy", 7))
        d["new_leaves"] = np.asarray(m.predict_leaf_assignments(Xn))
        ti, ts = m.predict_top_k_similar(Xn, 8)
        d["new_topk_idx"], d["new_topk_sim"] = np.asarray(ti), np.asarray(ts)
        d["iseed"] = np.int32(12345)
        out[name] = d
    return out


def main():
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref is not built: run `make -C oracle ref`")
    out = {}
    for name, (task, kind, n, p, seed, kw) in CASES.items():
        X, y = synth(kind, n, p, seed)
        r = oracle.ref_fit(task, X, y, **kw)
        d = {"X": X}
        if y is not None:
            d["y"] = y
        for k in KEYS:
            if r.get(k) is not None:
                d[k] = np.asarray(r[k])
        if kw.get("proximity"):
            N = r["nout"].shape[0]
            d["prox_pairs"] = r["prox_raw"].reshape(N, N).T.astype(np.int32)  # P[i][j]
            d["prox"] = r["prox"]
        d["maxnode"] = np.int32(r["maxnode"])
        out[name] = d
    # weighted bootstrap and binning vectors
    rng = np.random.default_rng(7)
    sw = rng.uniform(0.1, 3.0, size=900).astype(np.float32)
    boot = {"nin_w": np.stack([oracle.ref_bootstrap(900, t, sw) for t in range(3)]),
            "nin": np.stack([oracle.ref_bootstrap(900, t) for t in range(3)]), "sw": sw}
    Xb, cat = binning_data()
    e, nb, kind, xb = oracle.ref_binning(Xb, cat, 256)
    e16, nb16, kind16, xb16 = oracle.ref_binning(Xb, cat, 16)
    binning = {"X": Xb, "cat": cat, "edges": e, "nb": nb, "kind": kind, "xb": xb,
               "edges16": e16, "nb16": nb16, "kind16": kind16, "xb16": xb16}
    out.update(predict_golden())
    # an unsupervised model file (RandomForestUnsupervised.save)
    Xu, _ = synth("gmm", 300, 6, 5)
    u = oracle.ref_module().RandomForestUnsupervised(nsample=300, ntree=2, mtry=2, minndsize=1,
                                                     show_progress=False)
    u.fit(Xu)
    save_gz(u, os.path.join(HERE, "unsup_model.rfx.gz"))
    out["unsup_model"] = {"X": Xu}
    out["impute"] = impute_golden()
    out["impute_median"] = impute_golden("median")
    for name, d in out.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
    np.savez_compressed(os.path.join(HERE, "bootstrap.npz"), **boot)
    np.savez_compressed(os.path.join(HERE, "binning.npz"), **binning)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "leaves":  # only the leaf-query fixtures
        for name, d in leaves_golden().items():
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
    elif len(sys.argv) > 1 and sys.argv[1] == "impute":  # only the imputation fixtures
        for agg, name in (("mean", "impute"), ("median", "impute_median")):
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **impute_golden(agg))
    else:
        main()
