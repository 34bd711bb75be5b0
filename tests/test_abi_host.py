"""CPU-only checks of the boundary: the C-ABI library loads and exports every function
declared in include/rfx_b200.h, and the estimator wrappers resolve their arguments the way
the reference's wrappers do (python/randomforest_py.cpp)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import rfx_b200
from rfx_b200 import _abi as A
from rfx_b200.forest import _argmax_last, _isqrt_f32

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rfx_b200.h")


def declared_functions():
    src = open(os.path.join(ROOT, "include", "rfx_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rfx_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(A.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(A.SYMBOLS) <= set(names) | {"rfx_prox_dense_static"}


def test_abi_version_and_no_device_here_is_reported():
    lib = rfx_b200.load_library()
    with open(HEADER) as f:
        want = int(re.search(r"#define RFX_ABI_VERSION (\d+)", f.read()).group(1))
    assert lib.rfx_abi_version() == want
    assert lib.rfx_device_count() >= 0


def test_block_cache_is_empty_without_contexts():
    # nothing has been cached in a process that made no device context; emptying is a no-op
    assert rfx_b200.cached_bytes() == 0
    rfx_b200.empty_cache()
    assert rfx_b200.cached_bytes(0) == 0


def test_create_on_missing_device_fails_cleanly():
    lib = rfx_b200.load_library()
    h = lib.rfx_create(10_000)
    assert not h
    assert lib.rfx_last_error()


def test_calculate_maxnode_rule():
    # include/rf_config.hpp:15-32
    assert rfx_b200.calculate_maxnode(1000, 1) == 2001
    assert rfx_b200.calculate_maxnode(200_000, 5) == 32001
    assert rfx_b200.calculate_maxnode(10_000, 1) == 20001
    assert rfx_b200.calculate_maxnode(10_000, 0) == 20001
    assert rfx_b200.calculate_maxnode(10, 3, 77) == 77


def test_estimator_defaults_follow_the_reference_wrappers():
    # mtry=0 resolves from the constructor's mdim (default 10 -> 3) for classifier and
    # regressor alike; maxnode from the constructor's nsample (default 1000 -> 2001)
    c = rfx_b200.RandomForestClassifier()
    r = rfx_b200.RandomForestRegressor()
    assert c._mtry == 3 and r._mtry == 3
    assert c._maxnode == 2001 and r._maxnode == 2001
    assert rfx_b200.RandomForestClassifier(nsample=10_000, minndsize=1)._maxnode == 20001
    assert _isqrt_f32(50) == 7 and _isqrt_f32(16) == 4
    u = rfx_b200.RandomForestUnsupervised(mtry=0)
    assert u._mtry == 0  # resolved at fit time from the data (setup_unsupervised_task)


def test_unsupported_options_raise():
    with pytest.raises(NotImplementedError):
        rfx_b200.RandomForestClassifier(use_casewise=True)
    with pytest.raises(NotImplementedError):
        rfx_b200.RandomForestClassifier(use_rfgap=True)


def test_categorical_detection_rule():
    rng = np.random.default_rng(0)
    X = np.stack([rng.normal(size=500), rng.integers(0, 2, 500), rng.integers(0, 6, 500),
                  rng.integers(0, 12, 500), rng.integers(0, 6, 500) + 0.5]).T.astype(np.float32)
    cat = rfx_b200.detect_categorical(X, maxcat=10)
    assert cat.tolist() == [1, 1, 6, 1, 1]
    assert rfx_b200.detect_categorical(X, 10, [1]).tolist() == [1, 2, 1, 1, 1]


def test_oob_argmax_ties_go_to_the_last_class():
    q = np.array([[1, 1, 0], [0, 2, 2], [3, 1, 1]], np.float32)
    assert _argmax_last(q).tolist() == [1, 2, 0]


def test_rank_scores_desc_is_a_descending_sort():
    """compute_outliers' ranking (host only): descending scores, first k; distinct scores
    give the unique order, equal scores stay within their run."""
    rng = np.random.default_rng(11)
    s = rng.permutation(200).astype(np.float32) / np.float32(7.0)
    idx, val = A.rank_scores_desc(s, 15)
    ref = np.argsort(-s, kind="stable")[:15]
    assert np.array_equal(idx, ref) and np.array_equal(val, s[ref])
    t = np.repeat(np.arange(10, dtype=np.float32), 20)
    idx, val = A.rank_scores_desc(t, 50)
    assert np.all(np.diff(val) <= 0) and np.array_equal(val, t[idx])
    assert len(set(idx.tolist())) == 50
    idx, val = A.rank_scores_desc(s[:5], 9)
    assert idx.shape == (5,)


def test_task_type_and_aliases():
    """get_task_type (the reference's TaskType values) and the compute_proximity_matrix alias."""
    assert [int(t) for t in rfx_b200.TaskType] == [0, 1, 2]
    assert rfx_b200.RandomForestClassifier().get_task_type() == rfx_b200.TaskType.CLASSIFICATION
    assert rfx_b200.RandomForestRegressor().get_task_type() == rfx_b200.TaskType.REGRESSION
    assert rfx_b200.RandomForestUnsupervised().get_task_type() == rfx_b200.TaskType.UNSUPERVISED
    for cls in (rfx_b200.RandomForestClassifier, rfx_b200.RandomForestRegressor,
                rfx_b200.RandomForestUnsupervised):
        assert callable(cls.compute_proximity_matrix) and cls().cleanup() is None
