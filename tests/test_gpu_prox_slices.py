"""Finishing reduce-scattered slices of the packed proximity triangle (rfx_prox_finish_packed,
the per-rank step of a tree-sharded fit's combine) equals the dense finishprox'd matrix of
the same counts bit for bit, for slices that start and end inside rows."""
import numpy as np
import pytest

from _helpers import gpu_fit, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [1, 2, 3, 7])
def test_packed_slices_equal_dense(world):
    import torch

    from rfx_b200.shard import prox_slice
    X, y = synth("class", 1500, 8, 41)
    g = gpu_fit(0, X, y, ntree=9, mtry=3, minndsize=1, maxnode=3001, proximity=True)
    ctx = g["ctx"]
    R = X.shape[0]
    dense = g["prox"]
    iu = np.triu_indices(R, 1)
    want = dense[iu]
    dev, length = ctx.prox_buffer()
    nout_dev, _ = ctx.vote_buffers()
    assert length == len(want)
    got = np.empty(length, np.float32)
    for rank in range(world):
        e0, cnt, padded = prox_slice(length, rank, world)
        assert padded % world == 0 and padded >= length
        out = torch.empty(max(cnt, 1), dtype=torch.float32, device="cuda:0")
        torch.cuda.synchronize()
        ctx.prox_finish_packed(int(dev) + 4 * e0, e0, cnt, nout_dev, R, out.data_ptr())
        got[e0:e0 + cnt] = out[:cnt].cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
