#!/usr/bin/env python
"""Forest-growth throughput on BASELINE config[1] (one JSON line on stdout, rank 0).

Workload: regression, n=200,000 rows x p=50 float32 features
~ U(-1,1); y = sum_{j<10} sin(3 x_j) + 0.5 x_10 x_11 + N(0, 0.1^2); mtry=16, nodesize 5
(the reference's minndsize=5), 256 quantile bins, MSE splits, OOB error and permutation
importance, no proximity; maxnode = calculate_maxnode(n, 5) = 32001 (nsample=n passed).
Synthetic data, seeded (numpy default_rng(20261201 + 1)).

A step fits config[1]'s whole 500-tree forest on the device-resident dataset: the trees are
split over the N GPUs (rank r grows the id block [r*500/N, (r+1)*500/N), strong scaling),
then the forest-level results are combined across the ranks inside the timed region (OOB
counts all-reduced, the OOB prediction sums folded in tree order rank by rank, importance
rows gathered and summed in tree order).  Metric: fit trees/s for the whole job.

  value  device-resident: dataset loaded and binned in HBM before timing; CUDA events on the
         library's stream; max over ranks.  "checksum" hashes the combined arrays, so runs
         at different N can be compared (they are bit-identical).
  e2e    the public API a user calls: RandomForestRegressor(ntree=500).fit(X, y) (N > 1:
         rfx_b200.shard.fit_sharded) from pinned host X/y, including the upload and binning,
         the tree arrays' download and the combine, every step.
  proximity  the proximity half of the metric, from a config[0] forest (100 trees, OOB x
         in-bag counts + finishprox) in the same invocation (rank 0).

--impl reference times the reference's own CPU implementation (oracle/_ref, compiled from
the reference sources; else the CPU port) on the same workload with all host threads: each
step is one fit of --ref-step-trees trees, and the per-tree rate excludes the one-time
prepare_data (measured by a 1-tree fit and reported separately).

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


# DRAM bytes (read + write) of the histogram kernels per tree level (the unit the bench's
# histogram time and algorithmic bytes are counted in), measured once with ncu over every
# histogram launch of a 250-tree batch and carried here as a constant; the capture is
# summarised under profiles/.
HIST_TRAFFIC_BYTES = 179.6e6
HIST_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of every histogram "
                       "launch (k_hist_pipe, k_hist_lane, k_hist_lane_mid) of a 250-tree batch: "
                       "3232 MB over its 18 levels, per level, constant")


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


def cpu_tree_rate(X, y, k, fits=1):
    """Per-tree rate of the reference CPU fit excluding its one-time prepare_data: a 1-tree fit
    gives prepare + one tree, each k-tree fit adds k - 1 trees.  Returns (trees/s, prepare_s,
    kind, cores, [seconds of the k-tree fits], one-tree seconds)."""
    t1, kind, cores = cpu_reference_fit(X, y, 1)
    tk = []
    for _ in range(fits):
        dt, kind, cores = cpu_reference_fit(X, y, k)
        tk.append(dt)
    per_tree = (sum(tk) / len(tk) - t1) / (k - 1)
    rate = fits * (k - 1) / (sum(tk) - fits * t1)
    return rate, t1 - per_tree, kind, cores, tk, t1


def arm_config(trees):
    """The config both arms print (identical, so the two lines compare)."""
    return {"workload": WORKLOAD, "forest_trees": trees}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    X, y = make_data(CFG["n"], CFG["p"])
    k = max(2, args.ref_step_trees)
    t1, kind, cores = cpu_reference_fit(X, y, 1)  # prepare_data + one tree
    for _ in range(args.warmup):
        cpu_reference_fit(X, y, k)
    times = []
    for _ in range(args.steps):
        dt, kind, cores = cpu_reference_fit(X, y, k)
        times.append(dt)
    value = args.steps * (k - 1) / (sum(times) - args.steps * t1)
    prepare = t1 - (sum(times) / len(times) - t1) / (k - 1)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "trees/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * CFG["ntree"] / value, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": arm_config(CFG["ntree"]),
        "cpu_baseline": {"value": value, "unit": "trees/s", "cores": cores, "kind": kind,
                         "sample": f"{args.steps} fits of {k} trees on the full config[1] data; "
                                   f"per-tree rate = (k - 1) trees / (t_k - t_1) with t_1 a 1-tree "
                                   f"fit ({t1:.2f} s), so the one-time prepare_data "
                                   f"({prepare:.2f} s) is excluded",
                         "prepare_data_s": prepare, "fit_s": times},
        "e2e": {"value": value, "unit": "trees/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "details": {"ms_per_step_is": "time of the 500-tree forest at the measured per-tree rate"},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_rfx(args):
    if args.workload == "config1":
        return run_config1(args)
    from bench_workloads import run_workload
    return run_workload(args)


def run_config1(args):
    import hashlib

    import torch

    import rfx_b200
    from rfx_b200 import _abi as A
    from rfx_b200.shard import combine, fit_sharded, tree_block

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    n, p = CFG["n"], CFG["p"]
    X, y = make_data(n, p)
    M = calc_maxnode(n, CFG["minndsize"])
    T = args.forest_trees
    t0, t1 = tree_block(T, rank, world)
    k = t1 - t0
    ctx = rfx_b200.Context(local)
    prm = A.FitParams(A.TASK_REGRESSION, n, p, CFG["mtry"], CFG["minndsize"], M, 12345, 12345,
                      CFG["nbins"], 10, 1, 0, 0, args.batch_trees, 1)
    inp = A.Inputs(A.ptr(X, A._pf), None, A.ptr(y, A._pf), None, None, None)
    ctx.load(prm, inp)
    lib = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    rr = np.zeros((k, p), np.float32)
    used = np.zeros((k, p), np.uint8)
    trees = A.Trees(None, None, None, None, None, None, None, None, None, None,
                    A.ptr(rr, A._pf), A.ptr(used, A._pu8))
    with torch.cuda.stream(lib):
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

        def step():
            ctx.reset_forest()
            ctx.grow(t0, k, trees)
            acc, _ = combine(ctx, A.TASK_REGRESSION, n, p, 1, rr, used, dist, T, None, dev)
            return acc

        for _ in range(args.warmup):
            step()
        ctx.reset_stats()
        ctx.set_profiling(True)
        clocks = Clocks(local)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(lib)
        for _ in range(args.steps):
            flush.zero_()  # L2 flush between steps (256 MiB > 126 MB L2)
            acc = step()
        ev1.record(lib)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ck = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    st = ctx.stats()
    ctx.set_profiling(False)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = args.steps * T / (ms / 1000.0)
    h = hashlib.sha1()
    for key in ("nout", "oob_sum", "avimp", "sqsd"):
        h.update(np.ascontiguousarray(acc[key]).tobytes())
    checksum = h.hexdigest()[:16]

    # ---- e2e: the public estimator API with pinned host buffers
    Xp = torch.empty((n, p), dtype=torch.float32, pin_memory=True).numpy()
    yp = torch.empty((n,), dtype=torch.float32, pin_memory=True).numpy()
    Xp[:] = X
    yp[:] = y

    def e2e_fit():
        est = rfx_b200.RandomForestRegressor(nsample=n, ntree=T, mtry=CFG["mtry"],
                                             minndsize=CFG["minndsize"], compute_importance=True,
                                             device=local, batch_trees=args.batch_trees)
        if dist is not None:
            fit_sharded(est, Xp, yp, dist, local)
        else:
            est.fit(Xp, yp)
        return est.get_oob_error()

    e2e_fit()  # warm-up
    e2e_steps = max(1, args.e2e_steps)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ts = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_fit()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - ts
    if dist is not None:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = e2e_steps * T / e2e_s
    h2d = world * (Xp.nbytes + yp.nbytes + 4 * p)
    # what each fit copies back: node counts, per-tree importance rows (rr float + used
    # byte), nout and the OOB sums, avimp and sqsd (the tree arrays stay on the device)
    d2h = T * 4 + T * p * 5 + n * 4 * 2 + p * 8

    peak, peak_kind = measured_peaks()
    hist_s = st["hist_ms"] / 1000.0
    achieved = (st["hist_bytes"] / hist_s / 1e9) if hist_s > 0 else None
    per_level_bytes = st["hist_bytes"] / max(1, st["hist_launches"])
    line = {
        "metric": METRIC, "value": value, "unit": "trees/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy, config[1] shapes and distributions)",
        "config": arm_config(T),
        "checksum": checksum,
        "details": {"step": f"one {T}-tree forest: reset, grow this rank's block, combine",
                    "trees_this_rank": k,
                    "parallelism": f"trees sharded over {world} GPU(s) (strong scaling); "
                                   "combine: nout all-reduce, ordered OOB fold (send/recv "
                                   "chain), importance all-gather, on the library stream",
                    "l2": "flushed between steps (256 MiB write on the library stream)",
                    "batch_trees": args.batch_trees or "auto"},
        "e2e": {"value": e2e_value, "unit": "trees/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
                "call": ("rfx_b200.shard.fit_sharded(RandomForestRegressor(ntree=500), X, y)"
                         if world > 1 else "rfx_b200.RandomForestRegressor(ntree=500).fit(X, y)")
                        + " + get_oob_error()"},
        "gpu_launches": int(st["kernel_launches"]),
        "roofline": {"bound": "hbm", "kernel": "histogram search (k_hist_pipe + k_hist_lane_mid "
                                                "+ k_hist_lane, one tree level)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": (achieved / peak) if achieved else None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": HIST_TRAFFIC_BYTES,
                     "traffic_source": HIST_TRAFFIC_SOURCE,
                     "algorithmic_bytes_per_level": per_level_bytes,
                     "levels": int(st["hist_launches"]), "kernel_ms": st["hist_ms"],
                     "share_of_step": st["hist_ms"] / (ms * world) if ms else None},
        "clocks": ck,
    }
    if rank == 0 and not args.no_proximity:
        from bench_workloads import proximity_probe
        line["proximity"] = proximity_probe(local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, prep, kind, cores, tk, t1s = cpu_tree_rate(X, y, args.cpu_trees)
        line["cpu_baseline"] = {
            "value": rate, "unit": "trees/s", "cores": cores, "kind": kind,
            "sample": f"reference fits of 1 and {args.cpu_trees} trees on the full config[1] "
                      f"data ({t1s:.1f} s, {tk[0]:.1f} s): ({args.cpu_trees} - 1) trees / time "
                      f"difference, excluding the one-time prepare_data ({prep:.1f} s)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="rfx", choices=["rfx", "reference"])
    ap.add_argument("--step-trees", type=int, default=None)
    ap.add_argument("--batch-trees", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-trees", type=int, default=3)
    ap.add_argument("--ref-step-trees", type=int, default=4)
    ap.add_argument("--forest-trees", type=int, default=CFG["ntree"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-proximity", action="store_true")
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
