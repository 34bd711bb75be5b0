"""The reference's model file format RFX0 v1 (RandomForest::save / load,
src/rf_random_forest.cpp:5987-6270): read and write it, so models move both ways between the
reference (`RFXFuse.load`, `.save`) and this package.

Layout (native little-endian, packed): magic u32 0x52465830, version u32 1; the config
fields in the order of `FIELDS` (int32 / float32 / 1-byte bool / size_t-prefixed strings);
the sparse flag; then size_t-prefixed arrays: the tree arrays ([ntree x maxnode], treemap
x2, catgoleft [ntree x maxcat x maxnode]), nnode, cat, the importance arrays, leaf
assignments (int16), the per-sample OOB tree lists, the label map (size_t count of int32
pairs, then the reverse map), oob_error, oob_mse (float32) and nout.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = 0x52465830
VERSION = 1

# (name, kind) in file order; i = int32, f = float32, b = bool (1 byte), s = string
FIELDS = (
    ("nsample", "i"), ("ntree", "i"), ("mdim", "i"), ("nclass", "i"), ("maxcat", "i"),
    ("mtry", "i"), ("maxnode", "i"), ("minndsize", "i"), ("ncsplit", "i"), ("ncmax", "i"),
    ("iseed", "i"), ("task_type", "i"), ("compute_proximity", "b"), ("compute_importance", "b"),
    ("compute_local_importance", "b"), ("compute_proximity_importance", "b"),
    ("compute_leaf_assignments", "b"), ("use_rfgap", "b"), ("use_casewise", "b"),
    ("proximity_type", "s"), ("importance_method", "s"), ("clique_M", "i"), ("use_gpu", "b"),
    ("use_qlora", "b"), ("quant_mode", "i"), ("lowrank_rank", "i"),
    ("lowrank_power_iterations", "i"), ("use_sparse", "b"), ("sparsity_threshold", "f"),
    ("batch_size", "i"), ("use_histogram", "b"), ("n_bins", "i"), ("nodesize", "i"),
    ("cutoff", "f"), ("use_unsupervised", "b"), ("outlier_threshold", "f"),
    ("synthetic_ratio", "f"), ("unsupervised_mode", "i"), ("gpu_loss_function", "i"),
    ("n_threads_cpu", "i"),
)

# (name, dtype) of the arrays after the sparse flag, in file order
ARRAYS = (
    ("tnodewt", np.float32), ("nodepred", np.float32), ("xbestsplit", np.float32),
    ("nodestatus", np.int32), ("bestvar", np.int32), ("treemap", np.int32),
    ("catgoleft", np.int32), ("nodeclass", np.int32), ("nnode", np.int32), ("cat", np.int32),
    ("feature_importances", np.float32), ("avimp", np.float32), ("sqsd", np.float32),
    ("qimp", np.float32), ("qimpm", np.float32), ("proximity_importance", np.float32),
    ("leaf_assignments", np.int16),
)

_FMT = {"i": "<i", "f": "<f", "b": "<?"}


class _Reader:
    def __init__(self, data: bytes):
        self.d = data
        self.o = 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.d, self.o)[0]
        self.o += struct.calcsize(fmt)
        return v

    def size(self):
        return self.take("<Q")

    def string(self):
        n = self.size()
        s = self.d[self.o:self.o + n].decode()
        self.o += n
        return s

    def array(self, dtype):
        n = self.size()
        a = np.frombuffer(self.d, dtype=dtype, count=n, offset=self.o).copy()
        self.o += n * np.dtype(dtype).itemsize
        return a


def read(path: str) -> dict:
    """Parse an RFX0 file into a dict: config fields, arrays, `oob_trees` (list of int32
    arrays), `label_map` (list of (original, 0-based)), `label_inverse`, `oob_error`,
    `oob_mse`, `nout`."""
    with open(path, "rb") as f:
        r = _Reader(f.read())
    if r.take("<I") != MAGIC:
        raise RuntimeError(f"Invalid RFX model file (bad magic number): {path}")
    ver = r.take("<I")
    if ver != VERSION:
        raise RuntimeError(f"Unsupported RFX model version: {ver} (expected {VERSION})")
    m = {}
    for name, kind in FIELDS:
        m[name] = r.string() if kind == "s" else r.take(_FMT[kind])
    m["is_sparse"] = r.take("<?")
    for name, dt in ARRAYS:
        m[name] = r.array(dt)
    m["oob_trees"] = [r.array(np.int32) for _ in range(r.size())]
    m["label_map"] = [(r.take("<i"), r.take("<i")) for _ in range(r.size())]
    m["label_inverse"] = r.array(np.int32)
    m["oob_error"] = r.take("<f")
    m["oob_mse"] = r.take("<f")
    m["nout"] = r.array(np.int32)
    if r.o != len(r.d):
        raise RuntimeError(f"Error reading from file: {path} ({len(r.d) - r.o} trailing bytes)")
    return m


def write(path: str, m: dict) -> None:
    """Write a dict shaped like read()'s result as an RFX0 v1 file."""
    out = [struct.pack("<II", MAGIC, VERSION)]
    for name, kind in FIELDS:
        v = m[name]
        if kind == "s":
            b = str(v).encode()
            out.append(struct.pack("<Q", len(b)) + b)
        else:
            out.append(struct.pack(_FMT[kind], v))
    out.append(struct.pack("<?", bool(m.get("is_sparse", False))))

    def arr(a, dt):
        a = np.ascontiguousarray(np.asarray(a if a is not None else [], dtype=dt).ravel())
        out.append(struct.pack("<Q", a.size) + a.tobytes())

    for name, dt in ARRAYS:
        arr(m.get(name), dt)
    trees = m.get("oob_trees") or []
    out.append(struct.pack("<Q", len(trees)))
    for t in trees:
        arr(t, np.int32)
    lm = m.get("label_map") or []
    out.append(struct.pack("<Q", len(lm)))
    for a, b in lm:
        out.append(struct.pack("<ii", int(a), int(b)))
    arr(m.get("label_inverse"), np.int32)
    out.append(struct.pack("<ff", float(m.get("oob_error", 0.0)), float(m.get("oob_mse", 0.0))))
    arr(m.get("nout"), np.int32)
    with open(path, "wb") as f:
        f.write(b"".join(out))


# ---------------------------------------------------------------------------------------
# Estimators <-> model files
# ---------------------------------------------------------------------------------------
_QUANT = {"fp32": 0, "fp16": 1, "int8": 2, "nf4": 3}
_LOSS = {"gini": 0, "gini_impurity": 0, "mse": 3, "mean_squared_error": 3, "l2": 3}


def from_estimator(est) -> dict:
    """The fields RandomForest::save writes after the reference's own fit of the same model
    (config as the wrapper stores it, the tree arrays, importance, label maps, OOB results)."""
    from . import _abi as A
    task = est._task_id
    tr, acc = est.trees_, est.acc_
    T, M = tr["nodestatus"].shape
    p = est.n_features_
    nsample = est.n_rows_ if task == A.TASK_UNSUPERVISED else est.nsample
    m = {
        "nsample": nsample, "ntree": T, "mdim": p,
        "nclass": 1 if task == A.TASK_REGRESSION else est.nclass_,
        "maxcat": est.maxcat, "mtry": est._mtry_eff, "maxnode": M, "minndsize": est.minndsize,
        "ncsplit": est.ncsplit, "ncmax": est.ncmax, "iseed": est.iseed, "task_type": task,
        "compute_proximity": est.compute_proximity, "compute_importance": est.compute_importance,
        "compute_local_importance": False,
        "compute_proximity_importance": est.compute_proximity_importance,
        "compute_leaf_assignments": est.compute_leaf_assignments, "use_rfgap": False,
        "use_casewise": False, "proximity_type": "standard",
        "importance_method": est.importance_method, "clique_M": est.clique_M,
        "use_gpu": est.use_gpu, "use_qlora": est.use_qlora,
        "quant_mode": _QUANT.get(est.quant_mode.lower(), 3), "lowrank_rank": est.rank,
        "lowrank_power_iterations": est.power_iterations, "use_sparse": est.use_sparse,
        "sparsity_threshold": est.sparsity_threshold, "batch_size": est.batch_size,
        "use_histogram": True, "n_bins": est.n_bins, "nodesize": est.nodesize,
        "cutoff": est.cutoff, "use_unsupervised": False, "outlier_threshold": 2.0,
        "synthetic_ratio": est.synthetic_ratio, "unsupervised_mode": 0,
        "gpu_loss_function": 0 if task == A.TASK_UNSUPERVISED else _LOSS.get(est.gpu_loss_function.lower(), 0),
        "n_threads_cpu": est.n_threads_cpu, "is_sparse": False,
    }
    for k in ("tnodewt", "nodepred", "xbestsplit", "nodestatus", "bestvar", "treemap",
              "nodeclass", "nnode"):
        m[k] = tr[k]
    m["catgoleft"] = np.zeros(T * est.maxcat * M, np.int32)
    m["cat"] = est._cat
    if est.compute_importance:
        av = np.asarray(acc["avimp"], np.float32)
        s = np.add.accumulate(np.abs(av), dtype=np.float32)[-1] if len(av) else np.float32(0)
        m["feature_importances"] = av if s > 0 else np.zeros(p, np.float32)
        m["avimp"], m["sqsd"] = av, acc["sqsd"]
        m["qimp"] = np.zeros(nsample, np.float32)
    if task == A.TASK_CLASSIFICATION:
        m["label_map"] = [(int(c), i) for i, c in enumerate(est.classes_)]
        m["label_inverse"] = np.asarray(est.classes_, np.int32)
    m["oob_error"] = float(est._oob_error)
    m["oob_mse"] = float(est._oob_error) if task == A.TASK_REGRESSION else 0.0
    m["nout"] = acc["nout"]
    return m


class LoadedModel:
    """A model read from an RFX0 file (the reference's LoadedModel, python/randomforest_py.cpp:
    475-903): predict / predict_proba on the device, feature_importances_, save."""

    def __init__(self, m: dict, device: int = 0):
        from . import _abi as A
        self._m = m
        self._ctx = A.Context(device)
        T, M = m["ntree"], m["maxnode"]
        task = m["task_type"]
        if task not in (A.TASK_CLASSIFICATION, A.TASK_REGRESSION):
            self._loaded = False
            return
        trees = {k: np.asarray(m[k]).reshape(T, -1) for k in
                 ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodeclass")}
        trees["nodepred"] = np.asarray(m["nodepred"]).reshape(T, -1)
        self._ctx.load_forest(task, trees, m["cat"], nclass=max(m["nclass"], 1))
        self._loaded = True

    def get_task_type(self):
        from .forest import TaskType
        return TaskType(self._m["task_type"])

    def predict(self, X):
        from . import _abi as A
        m = self._m
        if not self._loaded:
            raise NotImplementedError("predict of a loaded unsupervised model is not implemented")
        X = np.ascontiguousarray(X, np.float32)
        if m["task_type"] == A.TASK_REGRESSION:
            return self._ctx.predict(X, 0)
        if X.shape[0] == m["nsample"]:
            # the training-size branch reads OOB predictions, which model files do not carry
            # (src/rf_random_forest.cpp:3384-3401): class 0 for every row
            return np.zeros(X.shape[0], np.int32)
        cls, _ = self._ctx.predict(X, m["nclass"])
        inv = m["label_inverse"]
        return (inv[cls] if len(inv) else cls).astype(np.int32)

    def predict_proba(self, X):
        m = self._m
        if not self._loaded:
            raise NotImplementedError("predict_proba of a loaded unsupervised model is not implemented")
        X = np.ascontiguousarray(X, np.float32)
        if X.shape[0] == m["nsample"]:
            return np.full((X.shape[0], m["nclass"]), np.float32(1.0 / m["nclass"]), np.float32)
        _, proba = self._ctx.predict(X, m["nclass"])
        return proba

    def feature_importances_(self):
        return np.asarray(self._m["feature_importances"], np.float32).copy()

    def get_n_features(self):
        return self._m["mdim"]

    def get_n_classes(self):
        return self._m["nclass"]

    def save(self, filepath):
        write(str(filepath), self._m)


def load(filepath: str, device: int = 0) -> LoadedModel:
    """RFXFuse.load (python/randomforest_py.cpp:897-903)."""
    return LoadedModel(read(str(filepath)), device)
