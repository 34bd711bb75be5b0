"""Multi-rank combine logic of tree-sharded fits, on CPU with gloo (world size 2 and 3).

The float folds must reproduce the single-process tree order exactly: regression OOB
prediction sums, importance sums; vote counts are integer sums; q is rebuilt from counts.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rfx_b200.shard import ordered_fold, ordered_importance, tree_block, votes_to_q

N, P, T = 257, 7, 11


def synthetic_trees():
    rng = np.random.default_rng(5)
    pred = rng.normal(size=(T, N)).astype(np.float32) * np.float32(3.7)
    pred[rng.random((T, N)) < 0.6] = np.nan          # in-bag rows of each tree
    rr = rng.normal(size=(T, P)).astype(np.float32) * np.float32(1e-3)
    used = (rng.random((T, P)) < 0.7).astype(np.uint8)
    cls = rng.integers(0, 3, size=(T, N))
    return pred, rr, used, cls


def serial_reference():
    pred, rr, used, cls = synthetic_trees()
    s = np.zeros(N, np.float32)
    for t in range(T):
        ok = ~np.isnan(pred[t])
        s[ok] = (s[ok] + pred[t][ok]).astype(np.float32)
    av = np.zeros(P, np.float32)
    sq = np.zeros(P, np.float32)
    for t in range(T):
        r = np.where(used[t] != 0, rr[t], 0).astype(np.float32)
        av = (av + r).astype(np.float32)
        sq = (sq + r * r).astype(np.float32)
    w = np.array([0.1, 0.7, 1.3], np.float32)
    q = np.zeros((N, 3), np.float32)
    votes = np.zeros((N, 3), np.int64)
    for t in range(T):
        oob = ~np.isnan(pred[t])
        idx = np.flatnonzero(oob)
        q[idx, cls[t, idx]] = (q[idx, cls[t, idx]] + w[cls[t, idx]]).astype(np.float32)
        votes[idx, cls[t, idx]] += 1
    return s, av, sq, q, votes, w


def worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pred, rr, used, cls = synthetic_trees()
    t0, t1 = tree_block(T, rank, world)

    def fold_local(v):
        a = v.numpy()
        for t in range(t0, t1):
            ok = ~np.isnan(pred[t])
            a[ok] = (a[ok] + pred[t][ok]).astype(np.float32)

    vec = torch.zeros(N, dtype=torch.float32)
    ordered_fold(vec, fold_local, dist)
    av, sq = ordered_importance(rr[t0:t1], used[t0:t1], dist)
    votes = np.zeros((N, 3), np.int64)
    for t in range(t0, t1):
        idx = np.flatnonzero(~np.isnan(pred[t]))
        votes[idx, cls[t, idx]] += 1
    tv = torch.from_numpy(votes)
    dist.all_reduce(tv)
    out[rank] = (vec.numpy().copy(), av, sq, tv.numpy().copy())
    dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_combine_matches_single_process_order(world):
    s, av, sq, q, votes, w = serial_reference()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(worker, args=(world, free_port(), out), nprocs=world, join=True)
    for r in range(world):
        vec, a, b, tv = out[r]
        assert np.array_equal(vec.view(np.uint32), s.view(np.uint32))
        assert np.array_equal(a.view(np.uint32), av.view(np.uint32))
        assert np.array_equal(b.view(np.uint32), sq.view(np.uint32))
        assert np.array_equal(tv, votes)
        assert np.array_equal(votes_to_q(tv, w).view(np.uint32), q.view(np.uint32))


def test_tree_blocks_partition_the_forest():
    for world in (1, 2, 3, 8):
        blocks = [tree_block(1000, r, world) for r in range(world)]
        assert blocks[0][0] == 0 and blocks[-1][1] == 1000
        assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))


@pytest.mark.parametrize("length", [0, 1, 10, 4950, 1_249_975_000])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_prox_slices_cover_the_triangle(length, world):
    from rfx_b200.shard import prox_slice
    ends = 0
    padded = None
    for r in range(world):
        e0, cnt, pad = prox_slice(length, r, world)
        assert e0 == ends or cnt == 0
        ends = e0 + cnt
        padded = pad if padded is None else padded
        assert pad == padded and pad % world == 0
        assert cnt <= pad // world
    assert ends == length and padded >= length
