"""rfx_prox_dense_static: the allocation-free proximity export.

Some callers cannot allocate device memory (a serving process or a host application whose
own pool owns the GPU's memory budget).  This entry point stages rows in a fixed device
array instead of cudaMalloc'd scratch; its output must equal rfx_prox_dense's, call after
call.  Kept in its own file so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from _helpers import gpu_fit, synth
from rfx_b200 import _abi as A

pytestmark = pytest.mark.gpu


def _entry():
    L = A.load_library()
    f = L.rfx_prox_dense_static
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                  C.POINTER(C.c_float), C.c_void_p]
    return f


def test_static_scratch_matches_allocating_path_twice():
    X, y = synth("class", 900, 8, 11)
    g = gpu_fit(0, X, y, ntree=5, mtry=3, minndsize=1, maxnode=1801, proximity=True)
    ctx = g["ctx"]
    upper, length = ctx.prox_buffer()
    nout_dev, _ = ctx.vote_buffers()
    R = 900
    assert length == R * (R - 1) // 2
    want = g["prox"]  # rfx_prox_dense (allocating path)
    f = _entry()
    out = np.full((R, R), np.nan, np.float32)
    rc = f(upper, nout_dev, R, 0, R, out.ctypes.data_as(C.POINTER(C.c_float)), ctx.stream())
    assert rc == 0, A.load_library().rfx_last_error()
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))
    # second call, another row range: the shared array keeps the first call's rows
    part = np.full((300, R), np.nan, np.float32)
    rc = f(upper, nout_dev, R, 250, 550, part.ctypes.data_as(C.POINTER(C.c_float)), None)
    assert rc == 0, A.load_library().rfx_last_error()
    assert np.array_equal(part.view(np.uint32), want[250:550].view(np.uint32))


def test_static_scratch_rejects_oversized_rows():
    X, y = synth("class", 300, 4, 12)
    g = gpu_fit(0, X, y, ntree=2, mtry=2, minndsize=1, maxnode=601, proximity=True)
    upper, _ = g["ctx"].prox_buffer()
    nout_dev, _ = g["ctx"].vote_buffers()
    out = np.zeros(4, np.float32)
    big = 4 * 1024 * 1024 + 1
    rc = _entry()(upper, nout_dev, big, 0, 1, out.ctypes.data_as(C.POINTER(C.c_float)), None)
    assert rc == -1  # RFX_ERR_ARG, before any device work
    assert b"exceeds the static scratch" in A.load_library().rfx_last_error()
