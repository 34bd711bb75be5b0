"""Proximity and low-rank workloads of bench.py (--workload config0 | config2 | config3).

Each prints one JSON line in bench.py's format.  A step grows `--step-trees` trees (default:
the configuration's whole forest for config0/config2, 125 trees -- one GPU's share of the
8-GPU config[3] run -- for config3) with the proximity work of that configuration; the
proximity counts are zeroed at the start of every step.  After the timed steps the
finishing stage is timed on its own: the dense finishprox'd matrix (config0/config2) or the
low-rank factor build and the top-50 of every row (config3).

Synthetic, seeded data with the shapes and distributions BASELINE.json gives.
"""
from __future__ import annotations

import json
import os
import time

import numpy as np

from bench import Clocks, Quiet, calc_maxnode, dist_env

WL = {
    "config0": dict(task=0, n=10_000, p=20, ntree=100, mtry=4, minndsize=1, seed=20261201,
                    prox_rows=0, lowrank=0,
                    workload="config[0]: classification n=10000 p=20 N(0,1), Bernoulli(sigmoid(x.w)) "
                             "labels, ntree=100, mtry=4, nodesize=1, OOB x in-bag proximity "
                             "(dense n x n) + importance"),
    "config2": dict(task=2, n=50_000, p=100, ntree=300, mtry=10, minndsize=1, seed=20261203,
                    prox_rows=50_000, lowrank=0,
                    workload="config[2]: unsupervised n=50000 real + 50000 synthetic rows, p=100 "
                             "5-component GMM, ntree=300, mtry=10, nodesize=1, proximity over the "
                             "50000 real rows"),
    "config3": dict(task=0, n=1_000_000, p=200, ntree=1000, mtry=14, minndsize=1, seed=20261204,
                    prox_rows=0, lowrank=64,
                    workload="config[3]: classification n=1000000 p=200 10-class GMM (30% noise "
                             "features), classwt [1..10]/10, mtry=14, nodesize=1, low-rank "
                             "proximity rank 64 (int8 factors) + top-50 per row"),
}


class _IntView:
    """Zero-copy view of `count` device int32 values for torch (CUDA array interface)."""

    def __init__(self, ptr, count):
        self.__cuda_array_interface__ = {"shape": (int(count),), "typestr": "<i4",
                                         "data": (int(ptr), False), "version": 3}


def make(cfg):
    rng = np.random.default_rng(cfg["seed"])
    n, p = cfg["n"], cfg["p"]
    if cfg is WL["config0"]:
        X = rng.normal(size=(n, p)).astype(np.float32)
        w = rng.normal(size=p)
        y = (rng.random(n) < 1.0 / (1.0 + np.exp(-(X @ w)))).astype(np.int32)
        return X, y, None
    if cfg is WL["config2"]:
        k = 5
        mu = rng.normal(scale=4.0, size=(k, p))
        var = rng.uniform(0.5, 2.0, size=(k, p))
        z = rng.integers(0, k, size=n)
        X = (mu[z] + rng.normal(size=(n, p)) * np.sqrt(var[z])).astype(np.float32)
        return X, None, None
    # config3: 10-class mixture, class means ~ N(0, 1.5^2) on 70% of the features, the
    # remaining 30% pure N(0, 1) noise, unit variance
    k, informative = 10, int(round(0.7 * p))
    mu = np.zeros((k, p), np.float32)
    mu[:, :informative] = rng.normal(scale=1.5, size=(k, informative))
    y = rng.integers(0, k, size=n).astype(np.int32)
    X = rng.standard_normal(size=(n, p), dtype=np.float32)
    X += mu[y]
    cw = (np.arange(1, 11) / 10.0).astype(np.float32)
    return X, y, cw


def peaks():
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def config4_data(seed=20261205):
    """n=100,000, p=40: 30 continuous N(0, Sigma) with pairwise correlation 0.4, 10 categorical
    with cardinality uniform in [2, 32]; 15% of cells missing completely at random."""
    rng = np.random.default_rng(seed)
    n = 100_000
    C = 0.4 * np.ones((30, 30)) + 0.6 * np.eye(30)
    L = np.linalg.cholesky(C)
    Xc = (rng.standard_normal((n, 30)) @ L.T).astype(np.float32)
    card = rng.integers(2, 33, size=10)
    Xk = np.stack([rng.integers(0, c, n) for c in card], axis=1).astype(np.float32)
    X = np.concatenate([Xc, Xk], axis=1)
    X[rng.random(X.shape) < 0.15] = np.nan
    return X


def run_impute(args):
    """config[4]: rfx_impute_proximity(X, ntree=200, n_iterations=5, mtry=6, minndsize=1)."""
    import torch

    import rfx_b200
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    X = config4_data()
    ntree, iters = 200, 5
    # warm-up: one short round on the same data
    rfx_b200.rfx_impute_proximity(X.copy(), ntree=8, n_iterations=1, mtry=6, minndsize=1,
                                  device=local)
    clocks = Clocks(local)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    Xo, info = rfx_b200.rfx_impute_proximity(X.copy(), ntree=ntree, n_iterations=iters, mtry=6,
                                             minndsize=1, device=local)
    torch.cuda.synchronize()
    total = time.perf_counter() - t0
    ck = clocks.stop()
    tim = info["timing_fit_fill_s"]
    rounds = len(tim)
    n_missing = int(np.isnan(X).sum())
    line = {
        "metric": "fit trees/sec (config4 imputation loop)", "value": rounds * ntree / total,
        "unit": "trees/s", "n_gpus": 1, "steps": rounds, "warmup": 1,
        "ms_per_step": 1000 * total / rounds, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32/int32",
        "data": "synthetic (seeded numpy, BASELINE config[4] shapes and distributions)",
        "config": {"workload": "config[4]: n=100000 p=40 (30 correlated continuous, 10 categorical "
                               "cardinality U[2,32]), 15% MCAR; rfx_impute_proximity ntree=200, "
                               "5 rounds, mtry=6, minndsize=1; unsupervised forests over 200000 "
                               "rows, proximity over the 100000 real rows",
                   "step": "one imputation round (fit + proximity + fill)"},
        "impute": {"missing_cells": n_missing, "rounds": rounds,
                   "fit_s": [round(a, 3) for a, _ in tim], "fill_s": [round(b, 3) for _, b in tim],
                   "total_s": total,
                   "fill_cells_per_s": n_missing / (sum(b for _, b in tim) / rounds)},
        "clocks": ck,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_workload(args):
    import torch
    if args.workload == "config4":
        return run_impute(args)

    import rfx_b200
    from rfx_b200 import _abi as A

    cfg = WL[args.workload]
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    X, y, cw = make(cfg)
    n, p, task = cfg["n"], cfg["p"], cfg["task"]
    N = 2 * n if task == 2 else n
    M = calc_maxnode(N, cfg["minndsize"])
    S = args.step_trees if args.step_trees_set else (125 if args.workload == "config3" else cfg["ntree"])
    ctx = rfx_b200.Context(local)
    prm = A.FitParams(task, n, p, cfg["mtry"], cfg["minndsize"], M, 12345, 12345, 256, 10,
                      int(args.workload == "config0"), 1, cfg["prox_rows"], args.batch_trees, 0,
                      cfg["lowrank"])
    inp = A.Inputs(A.ptr(X, A._pf), A.ptr(y, A._pi) if y is not None else None, None, None, None,
                   A.ptr(cw, A._pf) if cw is not None else None)
    ctx.load(prm, inp)
    R = cfg["prox_rows"] or N
    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    lowrank = cfg["lowrank"] > 0

    def step(tree0):
        if not lowrank:
            ctx.set_prox_buffer(None, R * (R - 1) // 2)  # zero the counts
        ctx.grow(tree0, S)

    next_tree = rank * 1_000_000
    for _ in range(args.warmup):
        if lowrank:
            ctx.load(prm, inp)  # keep only the timed trees in the low-rank store
        step(next_tree)
        next_tree += S
    if lowrank:
        ctx.load(prm, inp)
    ctx.reset_stats()
    ctx.set_profiling(True)
    clocks = Clocks(local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            flush.zero_()
            step(next_tree)
            next_tree += S
        ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ck = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    st = ctx.stats()
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = world * args.steps * S / (ms / 1000.0)
    hbm, bf16, peak_kind = peaks()
    line = {
        "metric": f"fit trees/sec ({args.workload})", "value": value, "unit": "trees/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32/int32",
        "data": "synthetic (seeded numpy, BASELINE shapes and distributions)",
        "config": {"workload": cfg["workload"], "step_trees": S,
                   "l2": "flushed between steps (256 MiB write on the library stream)"},
        "gpu_launches": int(st["kernel_launches"]), "clocks": ck,
    }
    if not lowrank:
        pairs = st["prox_pair_updates"]
        # finishprox of all R rows into a device buffer (reads the R(R-1)/2 counts, writes R^2)
        dense = torch.empty((R, R), dtype=torch.float32, device=dev)
        up, _ = ctx.prox_buffer()
        nout_dev, _ = ctx.vote_buffers()
        torch.cuda.synchronize()
        ctx.prox_finish(up, nout_dev, R, 0, R, dense.data_ptr())  # warm
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            f0.record(stream)
            ctx.prox_finish(up, nout_dev, R, 0, R, dense.data_ptr())
            f1.record(stream)
        torch.cuda.synchronize()
        fin_ms = f0.elapsed_time(f1)
        fin_bytes = 4.0 * R * (R - 1) / 2 + 4.0 * R * R + 4.0 * R
        del dense
        line["proximity"] = {
            "pair_updates_per_step": pairs / args.steps,
            "pair_updates_per_s": pairs / (ms / 1000.0),
            "kernel_pair_updates_per_s": pairs / (st["prox_ms"] / 1000.0) if st["prox_ms"] else None,
            "kernel_ms_per_step": st["prox_ms"] / args.steps,
            "rows": R, "counts_bytes": 4 * R * (R - 1) // 2,
            "finish": {"ms": fin_ms, "bytes": fin_bytes, "achieved_gbs": fin_bytes / fin_ms / 1e6,
                       "peak_gbs": hbm, "frac": fin_bytes / fin_ms / 1e6 / hbm,
                       "peak_source": peak_kind},
        }
        line["roofline"] = {"bound": "hbm", "kernel": "k_prox_finish (dense finishprox)",
                            "achieved": fin_bytes / fin_ms / 1e6, "peak": hbm, "unit": "GB/s",
                            "frac": fin_bytes / fin_ms / 1e6 / hbm, "traffic": None,
                            "peak_source": peak_kind}
    else:
        trees = ctx.stats()["trees"]
        ctx.reset_stats()
        reduce = nout_dev = None
        if world > 1:
            # sharded build: OOB counts and every sketch pass summed over the ranks (NCCL)
            from rfx_b200.shard import _DeviceFloats
            nd, _ = ctx.vote_buffers()
            nout_t = torch.empty(R, dtype=torch.int32, device=dev)
            torch.cuda.synchronize()
            nout_t.copy_(torch.as_tensor(_IntView(nd, R), device=dev))
            torch.distributed.all_reduce(nout_t)
            nout_dev = nout_t.data_ptr()

            def reduce(ptr, count):
                t = torch.as_tensor(_DeviceFloats(ptr, count), device=dev)
                torch.distributed.all_reduce(t)
                torch.cuda.synchronize(dev)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        t0 = time.perf_counter()
        ctx.lowrank_build(64, 16, 1, seed=12345, nout_dev=nout_dev, reduce=reduce)
        build_s = time.perf_counter() - t0
        st2 = ctx.stats()
        if world > 1:
            torch.distributed.barrier()
        t0 = time.perf_counter()
        rows_mine, idx, val = ctx.lowrank_topk_part(50, rank, world)
        r0, r1 = 0, len(rows_mine)
        topk_s = time.perf_counter() - t0
        if world > 1:
            tt = torch.tensor([build_s, topk_s], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
            build_s, topk_s = float(tt[0]), float(tt[1])
        st3 = ctx.stats()
        tiles = st3["topk_tiles"]
        flops = tiles * 2.0 * 128 * 256 * 64
        dense_flops = 2.0 * (r1 - r0) * (((R + 255) // 256) * 256) * 64
        topk_ms = st3["topk_ms"]
        sk_gbs = st2["sketch_bytes"] / st2["sketch_ms"] / 1e6 if st2["sketch_ms"] else None
        line["lowrank"] = {
            "trees": int(trees), "rank": 64, "oversample": 16, "passes": 3,
            "build_s": build_s, "sketch_ms": st2["sketch_ms"], "sketch_gbs": sk_gbs,
            "sketch_frac_hbm": sk_gbs / hbm if sk_gbs else None,
            "topk_s": topk_s, "topk_kernel_ms": topk_ms, "tiles": int(tiles),
            "tiles_dense": int(((r1 - r0 + 127) // 128) * ((R + 255) // 256)),
            "rows_this_rank": [r0, r1],
            "tensor_tflops_executed": flops / topk_ms / 1e9 if topk_ms else None,
            "tensor_frac_executed": flops / topk_ms / 1e9 / bf16 if topk_ms else None,
            "dense_equivalent_tflops": dense_flops / topk_ms / 1e9 if topk_ms else None,
            "peak_tflops": bf16, "peak_source": peak_kind,
            "check_row0": [int(v) for v in idx[0, :5]],
        }
        line["roofline"] = {"bound": "tensor", "kernel": "k_topk_tc (Q Q^T + fused top-50)",
                            "achieved": flops / topk_ms / 1e9 if topk_ms else None, "peak": bf16,
                            "unit": "TFLOP/s",
                            "frac": flops / topk_ms / 1e9 / bf16 if topk_ms else None,
                            "traffic": None, "peak_source": peak_kind,
                            "note": "executed MMA flops; tiles past every row's exact "
                                    "Cauchy-Schwarz stop are skipped"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "config0":
        line["cpu_baseline"] = cpu_config0(X, y, args.cpu_trees)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def proximity_probe(local):
    """The proximity half of the metric for bench.py's default line: config[0]'s 100-tree
    classification forest with OOB x in-bag proximity counts (one untimed warm-up forest, one
    timed), then finishprox of the 10000 x 10000 matrix into device memory."""
    import torch

    import rfx_b200
    from rfx_b200 import _abi as A
    cfg = WL["config0"]
    dev = torch.device("cuda", local)
    X, y, _ = make(cfg)
    n, p = cfg["n"], cfg["p"]
    M = calc_maxnode(n, cfg["minndsize"])
    ctx = rfx_b200.Context(local)
    prm = A.FitParams(0, n, p, cfg["mtry"], cfg["minndsize"], M, 12345, 12345, 256, 10, 0, 1, 0,
                      0, 0, 0)
    ctx.load(prm, A.Inputs(A.ptr(X, A._pf), A.ptr(y, A._pi), None, None, None, None))
    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    R = n
    ctx.grow(0, cfg["ntree"])
    ctx.reset_forest()
    ctx.reset_stats()
    ctx.set_profiling(True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        ctx.grow(0, cfg["ntree"])
        e1.record(stream)
    torch.cuda.synchronize()
    fit_ms = e0.elapsed_time(e1)
    st = ctx.stats()
    ctx.set_profiling(False)
    pairs = st["prox_pair_updates"]
    dense = torch.empty((R, R), dtype=torch.float32, device=dev)
    up, _ = ctx.prox_buffer()
    nout_dev, _ = ctx.vote_buffers()
    ctx.prox_finish(up, nout_dev, R, 0, R, dense.data_ptr())  # warm
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        ctx.prox_finish(up, nout_dev, R, 0, R, dense.data_ptr())
        f1.record(stream)
    torch.cuda.synchronize()
    fin_ms = f0.elapsed_time(f1)
    fin_bytes = 4.0 * R * (R - 1) / 2 + 4.0 * R * R + 4.0 * R
    hbm, _, peak_kind = peaks()
    ctx.close()
    return {
        "workload": cfg["workload"], "trees": cfg["ntree"], "fit_ms": fit_ms,
        "trees_per_s": cfg["ntree"] / (fit_ms / 1000.0),
        "pair_updates": pairs, "pair_updates_per_s": pairs / (fit_ms / 1000.0),
        "counting_ms": st["prox_ms"],
        "counting_pair_updates_per_s": pairs / (st["prox_ms"] / 1000.0) if st["prox_ms"] else None,
        "finish": {"kernel": "k_prox_finish", "rows": R, "ms": fin_ms, "bytes": fin_bytes,
                   "achieved_gbs": fin_bytes / fin_ms / 1e6, "peak_gbs": hbm,
                   "frac": fin_bytes / fin_ms / 1e6 / hbm, "peak_source": peak_kind},
    }


def cpu_config0(X, y, k):
    import oracle
    cores = os.cpu_count() or 1
    try:
        Rm = oracle.ref_module()
    except ImportError:
        Rm = None
    if Rm is not None:
        m = Rm.RandomForestClassifier(nsample=X.shape[0], ntree=k, mtry=4, minndsize=1,
                                      compute_importance=True, compute_proximity=True,
                                      show_progress=False)
        with Quiet():
            t = time.perf_counter()
            m.fit(X, y)
            dt = time.perf_counter() - t
        kind = "reference"
    else:
        t = time.perf_counter()
        oracle.fit(0, X, y, ntree=k, mtry=4, minndsize=1,
                   maxnode=calc_maxnode(X.shape[0], 1), proximity=True, dump_trees=False)
        dt = time.perf_counter() - t
        kind, cores = "port", 1
    return {"value": k / dt, "unit": "trees/s", "cores": cores, "kind": kind,
            "sample": f"one reference fit of {k} trees with proximity on the full config[0] data "
                      f"({dt:.1f} s)"}


def run_workload_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    if args.workload != "config0":
        print(json.dumps({"impl": "reference", "unavailable":
                          f"{args.workload}: the reference CPU proximity does not fit this host "
                          "(its dense n x n double matrix exceeds host memory)"}), flush=True)
        return 0
    cfg = WL["config0"]
    X, y, _ = make(cfg)
    k = args.ref_step_trees
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_config0(X, y, k)
        if i >= args.warmup:
            vals.append(k / r["value"])
    total = sum(vals)
    value = args.steps * k / total
    print(json.dumps({"impl": "reference", "metric": "fit trees/sec (config0)", "value": value,
                      "unit": "trees/s", "n_gpus": world, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "dtype": "f64", "data": "synthetic (seeded)",
                      "config": {"workload": cfg["workload"], "step_trees": k},
                      "cpu_baseline": {"value": value, "unit": "trees/s", "cores": r["cores"],
                                       "kind": r["kind"], "sample": r["sample"]},
                      "e2e": {"value": value, "unit": "trees/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)
    return 0
