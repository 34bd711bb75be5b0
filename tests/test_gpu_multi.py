"""Tree-sharded fit over 2 GPUs (NCCL) equals the single-GPU fit bit for bit.
Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ngpu():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def worker(rank, world, port, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.join(os.path.dirname(here), "rfx-fuse_b200")]
    import torch
    import torch.distributed as dist
    import rfx_b200
    from rfx_b200.shard import fit_sharded
    from _helpers import synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    res = {}
    X, y = synth("regr", 2500, 10, 31)
    r = rfx_b200.RandomForestRegressor(nsample=2500, ntree=7, mtry=4, minndsize=3)
    fit_sharded(r, X, y, dist, rank)
    res["regr"] = (r.acc_["nout"], r.acc_["oob_sum"], r.acc_["avimp"], r.acc_["sqsd"],
                   np.float32(r.get_oob_error()))
    X, y = synth("class", 1500, 8, 32)
    c = rfx_b200.RandomForestClassifier(nsample=1500, ntree=5, mtry=3, minndsize=1,
                                        compute_proximity=True, classwt=[0.3, 1.0])
    fit_sharded(c, X, y, dist, rank)
    res["class"] = (c.acc_["nout"], c.acc_["q"], c.acc_["avimp"], np.float32(c.get_oob_error()),
                    c.get_proximity_matrix())
    X, y = synth("multiclass", 3000, 8, 33)
    L = rfx_b200.RandomForestClassifier(nsample=3000, ntree=8, mtry=3, minndsize=1,
                                        compute_proximity=True, compute_importance=False,
                                        use_qlora=True, quant_mode="int8", rank=16)
    fit_sharded(L, X, y, dist, rank)
    q, s = L.get_lowrank_quantized()
    idx, val = L.get_lowrank_topk(10)  # collective: rows split over the ranks
    res["lowrank"] = (q, s, idx, val)
    out[rank] = res
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_fit_equals_single_gpu():
    import torch.multiprocessing as mp

    import rfx_b200
    from _helpers import synth
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(worker, args=(2, port, out), nprocs=2, join=True)
    X, y = synth("regr", 2500, 10, 31)
    r = rfx_b200.RandomForestRegressor(nsample=2500, ntree=7, mtry=4, minndsize=3)
    r.fit(X, y)
    X2, y2 = synth("class", 1500, 8, 32)
    c = rfx_b200.RandomForestClassifier(nsample=1500, ntree=5, mtry=3, minndsize=1,
                                        compute_proximity=True, classwt=[0.3, 1.0])
    c.fit(X2, y2)
    want_r = (r.acc_["nout"], r.acc_["oob_sum"], r.acc_["avimp"], r.acc_["sqsd"], np.float32(r.get_oob_error()))
    want_c = (c.acc_["nout"], c.acc_["q"], c.acc_["avimp"], np.float32(c.get_oob_error()), c.get_proximity_matrix())
    # low-rank: identical factors on both ranks (the sketch is all-reduced), the gathered
    # top-k equals the single-GPU top-k of those factors, and the factors agree with a
    # single-GPU fit up to the order of the fp32 sums
    q0, s0, i0, v0 = out[0]["lowrank"]
    q1, s1, i1, v1 = out[1]["lowrank"]
    assert np.array_equal(q0, q1) and np.array_equal(s0, s1)
    assert np.array_equal(i0, i1) and np.array_equal(v0, v1)
    ctx = rfx_b200.Context(0)
    ctx.lowrank_set_factors(q0, s0)
    iw, vw = ctx.lowrank_topk(10, 0, q0.shape[0])
    assert np.array_equal(i0, iw) and np.array_equal(v0.view(np.uint32), vw.view(np.uint32))
    X3, y3 = synth("multiclass", 3000, 8, 33)
    L = rfx_b200.RandomForestClassifier(nsample=3000, ntree=8, mtry=3, minndsize=1,
                                        compute_proximity=True, compute_importance=False,
                                        use_qlora=True, quant_mode="int8", rank=16)
    L.fit(X3, y3)
    A1 = L.get_lowrank_factors()[0]
    A2 = s0[:, None].astype(np.float64) * q0.astype(np.float64)
    P1, P2 = A1 @ A1.T, A2 @ A2.T
    assert np.sqrt(np.mean((P1 - P2) ** 2)) < 1e-2 * np.abs(P1).max()
    for rank in range(2):
        for got, want in zip(out[rank]["regr"], want_r):
            assert np.array_equal(np.atleast_1d(got).view(np.uint8), np.atleast_1d(want).view(np.uint8))
        for got, want in zip(out[rank]["class"], want_c):
            assert np.array_equal(np.atleast_1d(got).view(np.uint8), np.atleast_1d(want).view(np.uint8))
