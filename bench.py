#!/usr/bin/env python
"""Forest-growth throughput on BASELINE config[1] (one JSON line on stdout, rank 0).

Workload: regression, n=200,000 rows x p=50 float32 features
~ U(-1,1); y = sum_{j<10} sin(3 x_j) + 0.5 x_10 x_11 + N(0, 0.1^2); mtry=16, nodesize 5
(the reference's minndsize=5), 256 quantile bins, MSE splits, OOB error and permutation
importance, no proximity; maxnode = calculate_maxnode(n, 5) = 32001 (nsample=n passed).
Synthetic data, seeded (numpy default_rng(20261201 + 1)).

A step grows `--step-trees` trees of that forest (bootstrap, level-wise growth, OOB drop,
OOB prediction fold, permutation importance).  Metric: fit trees/s for the whole job.

  value  device-resident: dataset loaded and binned in HBM before timing; each step is one
         rfx_grow call; CUDA events on the library's stream; max over ranks.
  e2e    the public API call a user makes, RandomForestRegressor(ntree=step_trees).fit(X, y),
         from pinned host X/y to host tree arrays and OOB results, every step.

--impl reference times the reference's own CPU implementation (oracle/_ref, compiled from
the reference sources; else the CPU port) on the same workload with all host threads.

Other workloads (--workload; each prints its own line, the default is config1):
  config0  classification n=10000 p=20, 100 trees, mtry 4, nodesize 1, OOB x in-bag proximity
           counts + finishprox'd dense matrix; adds "proximity" (pair updates/s, finish GB/s).
  config2  unsupervised n=50000 real rows (+50000 synthetic) p=100 GMM, 300 trees, mtry 10,
           nodesize 1, proximity counts over the 50000 real rows (5 GB upper triangle).
  config3  classification n=1,000,000 p=200 10-class GMM, classwt [1..10]/10, mtry 14,
           nodesize 1, low-rank proximity rank 64 (int8 factors) + top-50 per row; adds
           "lowrank" (sketch GB/s, product TFLOP/s on the tensor cores, top-50 time).
  config4  the imputation loop rfx_impute_proximity (n=100000 p=40, 15% missing, 5 rounds of
           200-tree unsupervised forests with proximity and the device fill).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rfx-fuse_b200"))
sys.path.insert(0, ROOT)

CFG = dict(n=200_000, p=50, ntree=500, mtry=16, minndsize=5, nbins=256)
METRIC = "fit trees/sec (config[1] regression forest)"
WORKLOAD = ("config[1]: regression n=200000 p=50 U(-1,1), ntree=500 forest, mtry=16, "
            "nodesize(minndsize)=5, 256 bins, MSE splits, OOB error + permutation importance, "
            "no proximity, maxnode=32001")


def make_data(n, p, seed=20261201 + 1):
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1.0, 1.0, size=(n, p)).astype(np.float32)
    y = np.sin(3.0 * X[:, :10]).sum(axis=1) + 0.5 * X[:, 10] * X[:, 11]
    y = (y + rng.normal(0.0, 0.1, size=n)).astype(np.float32)
    return X, y


def calc_maxnode(n, m):
    return min(2 * ((n + m - 1) // m) + 1, 32001)


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, r[4:8]):
                if v.strip().lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic():
    """Per-launch DRAM traffic of the histogram kernels from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "k_hist_config1.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_level_full:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class Quiet:
    """Silence C-level stdout (the reference prints banners) while keeping our JSON clean."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        self.null = os.open(os.devnull, os.O_WRONLY)
        os.dup2(self.null, 1)

    def __exit__(self, *a):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.null)
        os.close(self.saved)


def cpu_reference_fit(X, y, ntree):
    """One fit of the reference CPU implementation; returns (seconds, kind, cores)."""
    import oracle
    cores = os.cpu_count() or 1
    try:
        R = oracle.ref_module()
    except ImportError:
        R = None
    if R is not None:
        m = R.RandomForestRegressor(nsample=X.shape[0], ntree=ntree, mtry=CFG["mtry"],
                                    minndsize=CFG["minndsize"], compute_importance=True,
                                    compute_proximity=False, show_progress=False)
        with Quiet():
            t = time.perf_counter()
            m.fit(X, y)
            dt = time.perf_counter() - t
        return dt, "reference", cores
    t = time.perf_counter()
    oracle.fit(1, X, y, ntree=ntree, mtry=CFG["mtry"], minndsize=CFG["minndsize"],
               maxnode=calc_maxnode(X.shape[0], CFG["minndsize"]), dump_trees=False)
    return time.perf_counter() - t, "port", 1


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    X, y = make_data(CFG["n"], CFG["p"])
    k = args.ref_step_trees
    for _ in range(args.warmup):
        cpu_reference_fit(X, y, k)
    times = []
    kind = cores = None
    for _ in range(args.steps):
        dt, kind, cores = cpu_reference_fit(X, y, k)
        times.append(dt)
    total = sum(times)
    value = args.steps * k / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "trees/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "step_trees": k},
        "cpu_baseline": {"value": value, "unit": "trees/s", "cores": cores, "kind": kind,
                         "sample": f"{args.steps} fits of {k} trees each on the full config[1] data "
                                   "(each fit includes the reference's one-time prepare_data)"},
        "e2e": {"value": value, "unit": "trees/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_rfx(args):
    if args.workload == "config1":
        return run_config1(args)
    from bench_workloads import run_workload
    return run_workload(args)


def run_config1(args):
    import torch

    import rfx_b200
    from rfx_b200 import _abi as A

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    n, p = CFG["n"], CFG["p"]
    X, y = make_data(n, p)
    M = calc_maxnode(n, CFG["minndsize"])
    S = args.step_trees
    ctx = rfx_b200.Context(local)
    prm = A.FitParams(A.TASK_REGRESSION, n, p, CFG["mtry"], CFG["minndsize"], M, 12345, 12345,
                      CFG["nbins"], 10, 1, 0, 0, args.batch_trees, 0)
    inp = A.Inputs(A.ptr(X, A._pf), None, A.ptr(y, A._pf), None, None, None)
    ctx.load(prm, inp)
    stream = torch.cuda.ExternalStream(ctx.stream(), device=torch.device("cuda", local))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")
    # weak scaling: every rank grows its own trees, with distinct tree ids
    next_tree = rank * 1_000_000
    for _ in range(args.warmup):
        ctx.grow(next_tree, S)
        next_tree += S
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
            flush.zero_()  # L2 flush between steps (256 MiB > 126 MB L2)
            ctx.grow(next_tree, S)
            next_tree += S
        ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ck = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    st = ctx.stats()
    ctx.set_profiling(False)
    if world > 1:
        t = torch.tensor([ms], device=f"cuda:{local}", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = world * args.steps * S / (ms / 1000.0)

    # ---- e2e: the public estimator API with pinned host buffers
    Xp = torch.empty((n, p), dtype=torch.float32, pin_memory=True).numpy()
    yp = torch.empty((n,), dtype=torch.float32, pin_memory=True).numpy()
    Xp[:] = X
    yp[:] = y
    est = rfx_b200.RandomForestRegressor(nsample=n, ntree=S, mtry=CFG["mtry"],
                                         minndsize=CFG["minndsize"], compute_importance=True,
                                         device=local, batch_trees=args.batch_trees)
    est.fit(Xp, yp)  # warm-up
    e2e_steps = max(1, args.e2e_steps)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        est.fit(Xp, yp)
        _ = est.get_oob_error()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=f"cuda:{local}", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = world * e2e_steps * S / e2e_s
    h2d = Xp.nbytes + yp.nbytes + 4 * p
    d2h = S * M * 4 * 9 + S * 4 + S * p * 5 + n * 4 * 2 + p * 8

    peak, peak_kind = measured_peaks()
    hist_s = st["hist_ms"] / 1000.0
    achieved = (st["hist_bytes"] / hist_s / 1e9) if hist_s > 0 else None
    per_level_bytes = st["hist_bytes"] / max(1, st["hist_launches"])
    line = {
        "metric": METRIC, "value": value, "unit": "trees/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy, config[1] shapes and distributions)",
        "config": {"workload": WORKLOAD, "step_trees": S, "trees_per_rank_timed": args.steps * S,
                   "parallelism": f"trees sharded over {world} GPU(s), no collective in the step",
                   "l2": "flushed between steps (256 MiB write on the library stream)",
                   "batch_trees": args.batch_trees or "auto"},
        "e2e": {"value": e2e_value, "unit": "trees/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
                "call": "rfx_b200.RandomForestRegressor(ntree=step_trees).fit(X, y) + get_oob_error()"},
        "gpu_launches": int(st["kernel_launches"]),
        "roofline": {"bound": "hbm", "kernel": "k_hist + k_hist_small (one tree level)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": (achieved / peak) if achieved else None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": profile_traffic(),
                     "algorithmic_bytes_per_level": per_level_bytes,
                     "levels": int(st["hist_launches"]), "kernel_ms": st["hist_ms"],
                     "share_of_step": st["hist_ms"] / ms if ms else None},
        "clocks": ck,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        k = args.cpu_trees
        dt, kind, cores = cpu_reference_fit(X, y, k)
        line["cpu_baseline"] = {"value": k / dt, "unit": "trees/s", "cores": cores, "kind": kind,
                                "sample": f"one reference fit of {k} trees on the full config[1] "
                                          f"data ({dt:.1f} s, includes one-time prepare_data)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="rfx", choices=["rfx", "reference"])
    ap.add_argument("--step-trees", type=int, default=None)
    ap.add_argument("--batch-trees", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--cpu-trees", type=int, default=8)
    ap.add_argument("--ref-step-trees", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="config1", choices=["config1", "config0", "config2", "config3", "config4"])
    args = ap.parse_args()
    args.step_trees_set = args.step_trees is not None
    if args.step_trees is None:
        args.step_trees = 250
    if args.impl == "reference" and args.workload != "config1":
        from bench_workloads import run_workload_reference
        return run_workload_reference(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_rfx(args)


if __name__ == "__main__":
    sys.exit(main())
