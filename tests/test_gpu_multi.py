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
    for rank in range(2):
        for got, want in zip(out[rank]["regr"], want_r):
            assert np.array_equal(np.atleast_1d(got).view(np.uint8), np.atleast_1d(want).view(np.uint8))
        for got, want in zip(out[rank]["class"], want_c):
            assert np.array_equal(np.atleast_1d(got).view(np.uint8), np.atleast_1d(want).view(np.uint8))
