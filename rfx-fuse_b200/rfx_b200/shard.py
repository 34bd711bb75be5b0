"""Tree-sharded fits over several GPUs (one process per GPU, torch.distributed).

Every tree's randomness depends only on its id (bootstrap MT19937(12345 + t), grower
MT19937(iseed + t)), so rank r grows the contiguous id block [r*T/W, (r+1)*T/W) and its
trees are identical to the single-GPU forest's.  Combining the ranks keeps the reference's
results exact:

* nout and the integer vote counts are summed (all-reduce); the classwt-weighted vote sums
  q are then rebuilt from the counts exactly as the reference accumulates them;
* regression OOB prediction sums are float sums in tree order, so they are folded rank by
  rank (rank r continues from rank r-1's vector) -- a chain of point-to-point transfers of
  one [N] vector, not a reduction;
* importance: per-tree rr rows are gathered and summed in tree order;
* proximity: integer counts in a caller-owned device buffer (the packed upper triangle),
  summed with one reduce-scatter into W equal slices; finishing is element-local (C_ij and
  the two row scales), so rank r finishes its own slice and the finished slices are gathered
  only when the dense matrix is asked for (get_proximity_matrix);
* low-rank proximity: every rank stores its own trees' leaf groups; each sketch pass applies
  the local trees to the block and the partial products are summed with one all-reduce
  (the library calls back between its passes), so every rank ends with the same factors;
  the top-k rows are then split over the ranks and gathered.

The collectives are plain torch.distributed calls (NCCL over NVLink on GPUs, gloo on CPU
for the tests), issued on the library's own CUDA stream so that they are ordered after its
kernels without host synchronisation; they run once per fit, outside the per-level work.
"""
from __future__ import annotations

import numpy as np


def tree_block(ntree: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous tree-id block of a rank: [begin, end)."""
    return ntree * rank // world, ntree * (rank + 1) // world


def ordered_fold(vec, fold_local, dist):
    """Fold a [N] float vector through the ranks in rank (= tree) order.

    ``vec`` starts at zero on every rank; ``fold_local(vec)`` adds this rank's trees in
    tree order, in place.  Returns the final vector on every rank.
    """
    rank, world = dist.get_rank(), dist.get_world_size()
    if rank > 0:
        dist.recv(vec, src=rank - 1)
    fold_local(vec)
    if rank < world - 1:
        dist.send(vec, dst=rank + 1)
    dist.broadcast(vec, src=world - 1)
    return vec


def prox_slice(length: int, rank: int, world: int) -> tuple[int, int, int]:
    """(first element, element count, padded length) of rank's slice of a packed triangle of
    ``length`` elements reduce-scattered into ``world`` equal slices (the padding past
    ``length`` holds zeros)."""
    per = -(-length // world) if length else 0
    e0 = min(length, rank * per)
    return e0, max(0, min(length, e0 + per) - e0), per * world


def ordered_importance(tree_rr: np.ndarray, tree_used: np.ndarray, dist, ntree=None, device=None):
    """avimp, sqsd = float32 sums over all ranks' trees in tree order (reference:
    src/rf_random_forest.cpp:1903-1906, avimp_[i] += avimp_temp[i] per tree).  The per-tree
    rows of every rank's block are gathered as tensors (blocks padded to the largest)."""
    import torch
    world, rank = dist.get_world_size(), dist.get_rank()
    rr_l = np.asarray(tree_rr, np.float32)
    used_l = np.asarray(tree_used, np.uint8)
    k, p = rr_l.shape
    T = ntree if ntree is not None else None
    if T is None:
        sizes = torch.tensor([k], dtype=torch.int64, device=device)
        allk = [torch.zeros_like(sizes) for _ in range(world)]
        dist.all_gather(allk, sizes)
        blocks = [int(a.item()) for a in allk]
    else:
        blocks = [tree_block(T, r, world)[1] - tree_block(T, r, world)[0] for r in range(world)]
    kmax = max(blocks)
    buf = torch.zeros((kmax, 2 * p), dtype=torch.float32, device=device)
    if k:
        buf[:k, :p] = torch.from_numpy(rr_l).to(buf.device)
        buf[:k, p:] = torch.from_numpy(used_l.astype(np.float32)).to(buf.device)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    g = [q.cpu().numpy() for q in parts]
    rr = np.concatenate([g[r][: blocks[r], :p] for r in range(world)])
    used = np.concatenate([g[r][: blocks[r], p:] for r in range(world)]) != 0
    return _fold_importance(rr, used)


def _fold_importance(rr: np.ndarray, used: np.ndarray):
    """avimp += rr, sqsd += rr^2 per tree, in tree order (float32); unused features add 0."""
    p = rr.shape[1]
    av = np.zeros(p, np.float32)
    sq = np.zeros(p, np.float32)
    for t in range(rr.shape[0]):
        r = np.where(used[t] != 0, rr[t], np.float32(0)).astype(np.float32)
        av = (av + r).astype(np.float32)
        sq = (sq + (r * r).astype(np.float32)).astype(np.float32)
    return av, sq


def votes_to_q(votes: np.ndarray, classwt) -> np.ndarray:
    """q[i][c] = classwt[c] added votes[i][c] times (float32, sequential).  Host version for
    the combine of a sharded fit; the device version is rfx_votes_to_q."""
    nclass = votes.shape[1]
    w = np.ones(nclass, np.float32) if classwt is None else np.asarray(classwt, np.float32)
    q = np.zeros(votes.shape, np.float32)
    kmax = int(votes.max()) if votes.size else 0
    for k in range(kmax):
        live = votes > k
        q = np.where(live, (q + w[None, :]).astype(np.float32), q)
    return q


class _DeviceFloats:
    """Zero-copy view of `count` device floats for torch (CUDA array interface)."""

    typestr = "<f4"

    def __init__(self, ptr: int, count: int):
        self.__cuda_array_interface__ = {"shape": (int(count),), "typestr": self.typestr,
                                         "data": (int(ptr), False), "version": 3}


class _DeviceInts(_DeviceFloats):
    """Zero-copy view of `count` device int32 values for torch."""

    typestr = "<i4"


def sharded_proximity_dense(est):
    """Dense finished proximity of a tree-sharded fit on every rank (collective): each rank
    finishes its reduce-scattered slice of the packed triangle on its GPU, the finished
    slices are gathered, and the matrix is assembled on the host (diagonal 1, mirrored)."""
    import torch
    sp = est._sharded_prox
    dist, part = sp["dist"], sp["counts"]
    world = dist.get_world_size()
    length, e0, cnt = sp["length"], sp["e0"], sp["count"]
    R = int(round((1 + (1 + 8 * length) ** 0.5) / 2)) if length else 1
    dev = part.device
    with torch.cuda.stream(sp["stream"]):
        fin = torch.zeros(part.numel(), dtype=torch.float32, device=dev)
        if cnt:
            est._context().prox_finish_packed(part.data_ptr(), e0, cnt, sp["nout"].data_ptr(), R,
                                              fin.data_ptr())
        parts = [torch.empty_like(fin) for _ in range(world)]
        dist.all_gather(parts, fin)
        vals = torch.cat(parts)[:length].cpu().numpy()
    out = np.zeros((R, R), np.float32)
    off = 0
    for i in range(R - 1):
        n_i = R - i - 1
        out[i, i + 1:] = vals[off:off + n_i]
        off += n_i
    B = 1024
    for i0 in range(0, R, B):
        i1 = min(R, i0 + B)
        out[i0:i1, :i0] = out[:i0, i0:i1].T
        blk = out[i0:i1, i0:i1]
        il = np.tril_indices(i1 - i0, -1)
        blk[il] = blk.T[il]
    np.fill_diagonal(out, 1.0)
    return out


def lowrank_topk_sharded(est, k: int, dist):
    """Top-k of all rows, split over the ranks by equal shares of the product kernel's row
    order (rfx_lowrank_topk_part; each rank works on its own GPU from the identical factors)
    and gathered: every rank returns the full result.  Collective: every rank must call it."""
    rank, world = dist.get_rank(), dist.get_world_size()
    rows, idx, val = est._context().lowrank_topk_part(int(k), rank, world)
    parts = [None] * world
    dist.all_gather_object(parts, (rows, idx, val))
    R = sum(len(p[0]) for p in parts)
    out_i = np.empty((R, k), np.int32)
    out_v = np.empty((R, k), np.float32)
    for r, i, v in parts:
        out_i[r] = i
        out_v[r] = v
    return out_i, out_v


def combine(ctx, task, N, p, ncl, rr, used, dist, ntree, classwt, dev, importance=True):
    """Forest-level results of every rank's trees, on every rank (collective; call it on the
    context's stream): nout and vote counts all-reduced and q rebuilt from the counts, or the
    regression OOB sums folded in tree order; importance summed in tree order from the
    gathered per-tree rows.  ``rr``/``used`` are this rank's per-tree importance rows.
    Returns (acc dict of host arrays, device nout tensor)."""
    import torch

    from . import _abi as A
    nout_dev, votes_dev = ctx.vote_buffers()
    t_nout = torch.as_tensor(_DeviceInts(nout_dev, N), device=dev).clone()
    if dist is not None:
        dist.all_reduce(t_nout)
    labels = np.zeros(N, np.int32)
    if ncl > 1:
        ctx.results(A.Accum(0, 0, None, None, None, None, None, None, A.ptr(labels, A._pi)))
    acc = {"labels": labels}
    if ncl > 1:
        t_votes = torch.as_tensor(_DeviceInts(votes_dev, N * ncl), device=dev).clone()
        if dist is not None:
            dist.all_reduce(t_votes)
        q = torch.zeros((N, ncl), dtype=torch.float32, device=dev)
        ctx.votes_to_q(t_votes.data_ptr(), classwt, N, ncl, q.data_ptr())
        acc["votes"] = t_votes.view(N, ncl).cpu().numpy()
        acc["q"] = q.cpu().numpy()
    else:
        vec = torch.zeros(N, dtype=torch.float32, device=dev)
        if dist is not None:
            ordered_fold(vec, lambda v: ctx.oob_fold(v.data_ptr()), dist)
        else:
            ctx.oob_fold(vec.data_ptr())
        acc["oob_sum"] = vec.cpu().numpy()
    acc["nout"] = t_nout.cpu().numpy()
    if importance:
        u = used if ncl > 1 else np.ones_like(used)
        if dist is not None:
            acc["avimp"], acc["sqsd"] = ordered_importance(rr, u, dist, ntree=ntree, device=dev)
        else:
            acc["avimp"], acc["sqsd"] = _fold_importance(np.asarray(rr, np.float32), u != 0)
    else:
        acc["avimp"] = acc["sqsd"] = np.zeros(p, np.float32)
    return acc, t_nout


def fit_sharded(est, X, y=None, dist=None, device=None):
    """Fit ``est`` (an rfx_b200 estimator) with its trees sharded over the process group.

    Every rank must call it with the same data.  Returns this rank's tree block; the
    estimator ends with the combined forest-level results (nout, votes/q or OOB sums,
    importance, proximity counts) on every rank.
    """
    import torch

    from . import _abi as A
    from .forest import (RandomForestClassifier, RandomForestRegressor, RandomForestUnsupervised,
                         _isqrt_f32, calculate_maxnode, feature_kinds)

    if dist is None:
        import torch.distributed as dist
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", device if device is not None else torch.cuda.current_device())
    X = np.ascontiguousarray(X, np.float32)
    n, p = X.shape
    if isinstance(est, RandomForestRegressor):
        task = A.TASK_REGRESSION
    elif isinstance(est, RandomForestUnsupervised):
        task = A.TASK_UNSUPERVISED
    elif isinstance(est, RandomForestClassifier):
        task = A.TASK_CLASSIFICATION
    else:
        raise TypeError("unsupported estimator")
    t0, t1 = tree_block(est.ntree, rank, world)
    # same preparation as est.fit, but grow only this rank's block
    if task == A.TASK_UNSUPERVISED:
        mtry = est._mtry if est._mtry > 0 else max(1, _isqrt_f32(p))
        maxnode = calculate_maxnode(2 * n, est.minndsize)
    else:
        mtry, maxnode = est._mtry, est._maxnode
    est.device = dev.index
    est._ctx = A.Context(dev.index)
    ctx = est._ctx
    cat = feature_kinds(task, X, est.maxcat, est.categorical_features)
    prm = A.FitParams(task, n, p, mtry, est.minndsize, maxnode, est.iseed, 12345, est.n_bins,
                      est.maxcat, int(est.compute_importance), int(est.compute_proximity),
                      est.prox_rows, est.batch_trees, int(task == A.TASK_REGRESSION),
                      est._lowrank_rank(), 0)
    ycls = np.ascontiguousarray(y, np.int32) if task == A.TASK_CLASSIFICATION else None
    yreg = np.ascontiguousarray(y, np.float32) if task == A.TASK_REGRESSION else None
    cw = None if getattr(est, "classwt", None) is None else np.ascontiguousarray(est.classwt, np.float32)
    inp = A.Inputs(A.ptr(X, A._pf), A.ptr(ycls, A._pi), A.ptr(yreg, A._pf), None,
                   A.ptr(cat, A._pi), A.ptr(cw, A._pf))
    ctx.load(prm, inp)
    N = 2 * n if task == A.TASK_UNSUPERVISED else n
    # every tensor operation and collective below runs on the library's stream
    lib = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    with torch.cuda.stream(lib):
        prox = None
        if est.compute_proximity and not est._lowrank_rank():
            _, length = ctx.prox_buffer()
            e0, cnt, padded = prox_slice(length, rank, world)
            prox = torch.zeros(padded, dtype=torch.int32, device=dev)
            ctx.set_prox_buffer(prox.data_ptr(), length)
        k = t1 - t0
        rr = np.zeros((k, p), np.float32)
        used = np.zeros((k, p), np.uint8)
        trees = A.Trees(None, None, None, None, None, None, None, None, None, None,
                        A.ptr(rr, A._pf), A.ptr(used, A._pu8))
        ctx.grow(t0, k, trees)
        ncl = 1 if task == A.TASK_REGRESSION else (2 if task == A.TASK_UNSUPERVISED else len(np.unique(ycls)))
        acc, t_nout = combine(ctx, task, N, p, ncl, rr, used, dist, est.ntree,
                              cw if task == A.TASK_CLASSIFICATION else None, dev,
                              importance=est.compute_importance)
        if prox is not None:
            part = torch.empty(padded // world, dtype=torch.int32, device=dev)
            dist.reduce_scatter_tensor(part, prox)
            # the full buffer stays alive: the context still holds its address
            est._sharded_prox = {"counts": part, "e0": e0, "count": cnt, "length": length,
                                 "nout": t_nout, "dist": dist, "stream": lib, "full": prox}
        if est._lowrank_rank():
            def reduce(ptr, count):
                t = torch.as_tensor(_DeviceFloats(ptr, count), device=dev)
                dist.all_reduce(t)

            ctx.lowrank_build(est.rank, est.lowrank_oversample, est.lowrank_power_iters,
                              seed=est.iseed, nout_dev=t_nout.data_ptr(), reduce=reduce)
            est._sharded_nout = t_nout  # keeps the device counts alive
            est._shard_dist = dist
        torch.cuda.current_stream(dev).synchronize()
    est.acc_ = acc
    est.n_rows_ = N
    est.nclass_ = ncl
    est.n_features_ = p
    est._fitted = True
    if task == A.TASK_REGRESSION:
        est._y = yreg
    est._finalize(y)
    return t0, t1
