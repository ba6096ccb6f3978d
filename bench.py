#!/usr/bin/env python
"""Benchmark of the YABT per-tree growth path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c4]

A step is one boosting iteration (gradients, level-wise tree growth, ridge-
linear neural leaves, interaction-score update, margin update) on the
configuration's synthetic data. The default workload is a 10,000,000 x 200
regression with correlated features (blocks of 10 columns, pairwise
correlation 0.3), 255 leaves, max depth 10, squared loss, neural leaves and
interaction steering on. Prints one JSON line.

value   trees/s over all GPUs with the inputs resident in HBM (CUDA events,
        max over ranks).
e2e     trees/s through the public estimator API (YABTRegressor.fit) from host
        memory: host->device copy of X and y, binning and K trees per fit.
impl=reference  the reference's own CPU implementation of the path (its OpenMP
        C grower yabt/_cgrow/grow.c and C apply, built under oracle/_ref, with
        interaction steering, plus the oracle restatement of its leaf models)
        on all host cores, on a 2,000,000-row sample, scaled to the workload.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

HIST_TRAFFIC_PER_ALG_BYTE = 3000.9 / 1548.1   # k_hist DRAM bytes per algorithmic byte (C4 shape, ncu)

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (n, F, leaves, max_depth, loss, lr)
    "c1": (20_000, 20, 31, 64, "mse", 0.1),
    "c2": (100_000, 50, 63, 64, "logloss", 0.05),
    "c3": (1_000_000, 100, 127, 64, "mse", 0.1),
    "c4": (10_000_000, 200, 255, 10, "mse", 0.1),
    "c5": (5_000_000, 128, 63, 64, "logloss", 0.1),
}


def workload_config(cfg: str, world: int) -> dict:
    """The ``config`` object of the JSON line (both arms)."""
    n, F, leaves, depth, loss, lr = CONFIGS[cfg]
    return {"workload": f"{cfg}: {n}x{F} sharded by rows over {world} GPU(s), {leaves} leaves, "
                        f"max_depth {depth}, {loss}, neural leaves, interaction steering",
            "global_rows": n, "rows_per_gpu": n // world,
            "l2": "inputs larger than L2 (bin matrix of C4: 2.08 GB)" if n * F > 10 ** 9 else "see workload",
            "parallelism": (f"row shards x{world}, level histograms summed by the NVLink exchange kernel"
                            if world > 1 else "one GPU")}


def make_data(cfg: str, n: int, F: int, device, seed: int = 0):
    """Seeded synthetic data with the configuration's shapes and distributions
    (generated on the device with torch's Philox generator)."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    if cfg == "c4":
        X = torch.randn(n, F, generator=g, device=device).mul_(0.7 ** 0.5)
        zb = torch.randn(n, F // 10, generator=g, device=device).mul_(0.3 ** 0.5)
        X.view(n, F // 10, 10).add_(zb.unsqueeze(2))
        del zb
        w = torch.randn(50, generator=g, device=device)
        y = torch.tanh(X[:, :50]) @ w
        for k in range(10):
            y += X[:, 2 * k] * X[:, 2 * k + 1]
        y += torch.randn(n, generator=g, device=device)
    elif cfg == "c1":
        X = torch.randn(n, F, generator=g, device=device)
        y = torch.sin(X[:, 0]) + X[:, 1] * X[:, 2] + 0.5 * X[:, 3] ** 2 + 0.2 * X[:, 4:10].sum(1)
        y += 0.1 * torch.randn(n, generator=g, device=device)
    elif cfg == "c3":
        X = torch.randn(n, F, generator=g, device=device)
        X[:, 80:] = torch.exp(X[:, 80:])
        w = torch.randn(20, generator=g, device=device)
        y = X[:, :20] @ w + 0.5 * X[:, 20] * X[:, 21] + 0.5 * torch.randn(n, generator=g, device=device)
        X[torch.rand(n, F, generator=g, device=device) < 0.05] = float("nan")
    elif cfg == "c5":   # 10 classes: argmax of linear scores + pair terms + Gumbel noise
        X = torch.randn(n, F, generator=g, device=device)
        X[torch.rand(n, F, generator=g, device=device) < 0.3] = 0.0
        W = torch.randn(F, 10, generator=g, device=device).mul_(0.3)
        sc = X @ W + 0.2 * X[:, :10] * X[:, 10:20]
        u = torch.rand(n, 10, generator=g, device=device).clamp_(1e-12, 1 - 1e-7)
        y = torch.argmax(sc - torch.log(-torch.log(u)), dim=1).float()
    else:   # c2: binary
        X = torch.randn(n, F, generator=g, device=device)
        logit = 0.8 * X[:, 0] - 0.5 * X[:, 1] + X[:, 2] * X[:, 3] + 0.3 * X[:, 4:15].sum(1)
        y = (torch.rand(n, generator=g, device=device) < torch.sigmoid(logit)).float()
    return X.contiguous(), y.contiguous()


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "20"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self, window: tuple[float, float] | None = None) -> dict:
        """Summary of the samples taken inside ``window`` (wall-clock seconds;
        all samples if none falls inside it)."""
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = [[c.strip() for c in ln.split(",")] for ln in open(self.f.name).read().strip().splitlines()
                if ln.strip()]
        os.unlink(self.f.name)
        rows = [r for r in rows if len(r) >= 10 and r[2].replace(".", "").isdigit()]

        def stamp(r):
            """Wall-clock seconds of an nvidia-smi timestamp, with or without a
            fractional part ("2026/12/02 06:23:01.123" or "... 06:23:01")."""
            try:
                whole, _, frac = r[0].partition(".")
                secs = time.mktime(time.strptime(whole.strip(), "%Y/%m/%d %H:%M:%S"))
                return secs + (float("0." + frac) if frac.strip().isdigit() else 0.0)
            except Exception:
                return None
        inside = rows
        if window is not None:
            sel = [r for r in rows if (t := stamp(r)) is not None and window[0] - 0.05 <= t <= window[1] + 0.05]
            if sel:
                inside = sel
        sm = [float(r[2]) for r in inside]
        mx = [float(r[3]) for r in inside if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i in range(4) if r[6 + i].lower() == "active"})
        load = [v for v in sm if v > 500] or sm
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(inside),
                "in_timed_region": len(inside) if inside is not rows else 0}


def cpu_reference(cfg: str, steps: int, warmup: int, threads: int, sample_rows: int, X_src=None, y_src=None):
    """The reference's CPU path on a row sample of the workload: per iteration,
    gradients, interaction steering (the reference steers for n >= 2000,
    yabt/boosting.py:339,410-412), its OpenMP C grower, its C apply, the leaf
    models (numpy restatement of yabt/neural_leaves.py:131-184; the reference's
    torch code cannot travel to the GPU box) and the margin update. ``warmup``
    untimed iterations, then the median of ``steps`` timed ones (trees 2..k of
    the fit when warmup is 1). Returns a dict: trees/s of the full workload
    (per-row cost x rows), seconds per sample step, ns per row, description."""
    from oracle import cgrow
    from oracle.binning import Binner as OBinner
    from oracle.boost import InteractionDetector
    n, F, leaves, depth, loss, lr = CONFIGS[cfg]
    if X_src is None:
        rng = np.random.default_rng(0)
        X = rng.standard_normal((sample_rows, F), dtype=np.float32)
        y = (np.tanh(X[:, :min(50, F)]) @ rng.standard_normal(min(50, F)).astype(np.float32)).astype(np.float32)
    else:
        X, y = X_src, y_src
    b = OBinner().fit(X)
    bins_fm = np.ascontiguousarray(b.transform(X).T)
    Xi = b.impute(X)
    margin = np.full(X.shape[0], float(y.mean()), np.float32)
    det = InteractionDetector(F) if X.shape[0] >= 2000 else None
    times = []
    for s in range(warmup + steps):
        dt, margin = cgrow.boosting_step_seconds(bins_fm, Xi, y, margin, b.edges_, leaves, depth, lr, threads,
                                                 detector=det)
        if s >= warmup:
            times.append(dt)
    per = statistics.median(times)
    m = X.shape[0]
    return {"trees_per_s": m / (n * per), "s_per_step": per, "ns_per_row": per / m * 1e9, "rows": m,
            "threads": threads,
            "desc": f"{m} of {n} rows x {F} features, {leaves} leaves, interaction steering, {threads} threads, "
                    f"median of {steps} iterations after {warmup}; trees/s = rows / (n x s per step)"}


def run_reference(args):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = args.config
    n, F, leaves, depth, loss, lr = CONFIGS[cfg]
    threads = os.cpu_count() or 1
    from oracle import cgrow
    if not cgrow.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libcgrow.so not built"}))
        return
    sample = min(n, args.ref_rows)
    X = y = None
    if torch.cuda.is_available():
        Xd, yd = make_data(cfg, sample, F, "cuda", seed=0)
        X, y = Xd.cpu().numpy(), yd.cpu().numpy()
    r = cpu_reference(cfg, args.steps, args.warmup, threads, sample, X, y)
    tps = r["trees_per_s"]
    line = {"impl": "reference", "metric": "trees_per_sec", "value": tps, "unit": "trees/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 / tps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(cfg, args.gpus),
            "sample_ms_per_step": 1000.0 * r["s_per_step"], "ns_per_row": r["ns_per_row"],
            "cpu_baseline": {"value": tps, "unit": "trees/s", "cores": threads, "kind": "reference",
                             "sample": r["desc"]},
            "e2e": {"value": tps, "unit": "trees/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def cpu_baseline_leg(cfg: str, dev) -> dict | None:
    """The reference's CPU path timed on this host for the JSON line's
    ``cpu_baseline``: all host cores at two sample sizes (the per-row cost of
    each shows whether scaling by rows holds), and the reference's default
    thread cap of 8 (yabt/grow_c.py:283-302) at the smaller one. The value is
    the larger sample at all cores."""
    from oracle import cgrow
    if not cgrow.available():
        return None
    n, F = CONFIGS[cfg][:2]
    cores = os.cpu_count() or 1
    runs = []
    for rows, threads in ((500_000, cores), (2_000_000, cores), (500_000, min(8, cores))):
        rows = min(rows, n)
        Xs, ys = make_data(cfg, rows, F, dev, seed=0)
        r = cpu_reference(cfg, 2, 1, threads, rows, Xs.cpu().numpy(), ys.cpu().numpy())
        del Xs, ys
        runs.append({k: r[k] for k in ("rows", "threads", "s_per_step", "ns_per_row", "trees_per_s")})
    main = runs[1]
    return {"value": main["trees_per_s"], "unit": "trees/s", "cores": main["threads"], "kind": "reference",
            "sample": f"{main['rows']} of {n} rows, interaction steering, median of 2 iterations after 1; "
                      "trees/s = rows / (n x s per step)",
            "os_cpu_count": cores, "omp_num_threads": os.environ.get("OMP_NUM_THREADS"), "runs": runs}


def run_multiclass(args):
    """C5: one-vs-rest over 10 classes, one tree per class per round, the class
    boosters interleaved on 10 CUDA streams (one GPU)."""
    import torch
    from yabt_b200 import _lib
    from yabt_b200.boosting import BoostParams
    from yabt_b200.multiclass import MulticlassBooster
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"metric": "trees_per_sec", "unavailable": "c5 (multiclass) runs on one GPU only"}))
        return
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    sampler = ClockSampler(0)
    sampler.start()
    n, F, leaves, depth, loss_name, lr = CONFIGS["c5"]
    lib = _lib.load()
    X, y = make_data("c5", n, F, dev, seed=1000)
    W, K = args.warmup, args.steps
    # one round after the timed ones: with the device-side level loop (whose
    # graph carries no events) the k_hist launches are timed in that round
    params = BoostParams(n_estimators=W + K + 1, max_leaves=leaves, max_depth=depth, learning_rate=lr)
    mc = MulticlassBooster(params)
    ev, marks = {}, {}

    def cb(r, streams):
        main = torch.cuda.current_stream()
        loop = mc.boosters_[0].grower_.level_loop_start() > 0
        marks["loop"] = loop
        if r == 0 and not loop:
            for b in mc.boosters_:
                b.grower_.set_timing(K * b.grower_.levels)
        if r == W - 1 or r == W + K - 1:
            for st in streams:
                main.wait_stream(st)
            e = torch.cuda.Event(enable_timing=True)
            e.record(main)
            ev["start" if r == W - 1 else "stop"] = e
            marks["l0" if r == W - 1 else "l1"] = int(lib.yabt_launch_count())
            if r == W - 1:
                marks["t0"] = time.time()
                for b in mc.boosters_:
                    if not loop:
                        b.grower_.set_timing(K * b.grower_.levels)
                    b.grower_.acc_reset()
                _lib.check(lib.yabt_launch_count_device_reset(_lib.stream_ptr()), "yabt_launch_count_device_reset")
                for st in streams:
                    st.wait_stream(main)
            else:
                marks["acc"] = [b.grower_.acc_read() for b in mc.boosters_]   # waits for the timed rounds
                marks["loop_launches"] = int(lib.yabt_launch_count_device())
                if loop:
                    for b in mc.boosters_:
                        b.grower_.set_timing(b.grower_.levels)      # the extra round, timed per launch
    torch.cuda.synchronize()
    mc.fit(X, y.cpu().numpy(), round_callback=cb)
    torch.cuda.synchronize()
    clocks = sampler.stop((marks["t0"], time.time()))
    ms = ev["start"].elapsed_time(ev["stop"])
    nc = len(mc.boosters_)
    hist_ms = sum(sum(b.grower_.hist_times()) for b in mc.boosters_)
    if marks["loop"]:
        hist_ms *= K                      # one round's k_hist time, for K rounds
    acc = marks["acc"]
    root, child, launches = (sum(a[i] for a in acc) for i in range(3))
    alg = root * (F + 8) + child * (F + 12)
    achieved = alg / (hist_ms / 1000.0) / 1e9 if hist_ms > 0 else float("nan")
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    # sparse-bin question (30% exact zeros per column): the shared-reduction
    # ceiling with every lane issuing, and with 30% of the lanes predicated off
    # as a histogram that skips each feature's default bin would issue them
    sink = torch.zeros(1, dtype=torch.int64, device=dev)
    probe = {}
    for active in (32, 31, 22, 8):
        rate = 0.0
        for _ in range(3):
            pms, pupd = ctypes.c_float(), ctypes.c_longlong()
            _lib.check(lib.yabt_probe_shared_red_masked(5, 400, active, sink.data_ptr(), _lib.stream_ptr(),
                                                        ctypes.byref(pms), ctypes.byref(pupd)), "probe")
            rate = max(rate, pupd.value / (pms.value / 1000.0) / 1e9)
        probe[f"active_{active}_of_32"] = rate
    # e2e through the public estimator API from pinned host memory: one
    # YABTClassifier fit of K rounds (host->device copy, binning, all classes)
    e2e = None
    if not args.no_e2e:
        from yabt_b200 import YABTClassifier
        Xh, yh = X.cpu().pin_memory(), y.cpu().numpy()
        del mc, X
        torch.cuda.empty_cache()
        kw = dict(max_leaves=leaves, max_depth=depth, learning_rate=lr)
        YABTClassifier(n_estimators=1, **kw).fit(Xh, yh)     # untimed warm-up fit of the same data
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        est = YABTClassifier(n_estimators=K, **kw).fit(Xh, yh)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        e2e = {"value": nc * K / dt, "unit": "trees/s",
               "h2d_bytes_per_step": int(n * (F + 1) * 4 / K),   # X and y once per fit, per round
               # each class booster reads back each tree's meta row and leaf-model flag
               "d2h_bytes_per_step": nc * (4 * 4 + 4),
               "fit_s": dt,
               "warmup": "one untimed fit of the same data and size before the timed fit",
               "stages_s": {k: round(v, 4) for k, v in
                            getattr(est.booster_, "fit_timings_", {}).items()}}
        del est, Xh
    print(json.dumps({
        "metric": "trees_per_sec", "value": nc * K / (ms / 1000.0), "unit": "trees/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded torch Philox, config shapes)",
        "config": {"workload": f"c5: {n}x{F}, {nc} classes one-vs-rest, one tree per class per round on "
                               f"{nc} CUDA streams, {leaves} leaves, logloss, neural leaves",
                   "global_rows": n, "l2": "inputs larger than L2"},
        "gpu_launches": marks["l1"] - marks["l0"] + marks.get("loop_launches", 0),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": "k_hist", "launches_timed": launches,
                     "concurrent_streams": nc,
                     "hist_time_source": "the round after the timed ones, CUDA events around each k_hist launch"
                     + (" (the timed rounds run their deeper levels in the device-side level loop)"
                        if marks["loop"] else ""),
                     "hist_launch_ms_over_step": hist_ms / ms,
                     "achieved_over_step": alg / (ms / 1000.0) / 1e9,
                     "how": f"achieved: k_hist's algorithmic bytes over the sum of its launch durations; the {nc} "
                            "class streams overlap, so each launch shares the GPU and the sum exceeds the step "
                            "(hist_launch_ms_over_step > 1); achieved_over_step: the same bytes over the step",
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650 GB/s"},
        "clocks": clocks, "e2e": e2e, "cpu_baseline": None,
        "sparse_bin_probe": {"unit": "G (row, feature) updates/s", "limbs": 5, **probe,
                             "how": "yabt_probe_shared_red_masked: k_hist's reductions alone, all lanes "
                                    "without a per-lane test (32), with it and 31, 22 (30% default-bin entries "
                                    "skipped) or 8 of 32 lanes issuing; updates/s count every (row, feature)"}}))


PHASE_TREES = 3      # trees grown after the timed ones with per-phase timing on


def phase_summary(phases, trees: int, dist, dev) -> dict:
    """Device time per tree of each phase of the library's launches, over the
    phase pass (the trees after the timed region, grown with CUDA events around
    every launch group; the max over ranks)."""
    import torch
    rec = phases.read()
    phases.stop()
    names = phases.names()
    t = torch.tensor([rec.get(n, {}).get("ms", 0.0) for n in names], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    per = {n: round(float(v) / trees, 4) for n, v in zip(names, t.tolist()) if v > 0}
    return {"ms_per_tree": per, "sum_ms_per_tree": round(sum(per.values()), 4), "trees": trees,
            "how": "CUDA events around every launch group of the library in trees grown after the timed "
                   "region (max over ranks); collective = host-issued NCCL all-reduces"}


def model_digest(booster, W: int, K: int, dist=None) -> dict:
    """SHA-256 over the timed trees (feature, threshold, left of trees W..W+K-1)
    and the root histogram's per-bin row counts summed over the ranks. Row
    shards change no split, count or partition, so the digest is the same at
    every GPU count."""
    import hashlib
    import torch
    h = hashlib.sha256()
    for t in booster.trees[W:W + K]:
        for a in (t.feature, t.threshold, t.left):
            h.update(a.detach().cpu().numpy().tobytes())
    counts = booster.grower_.root_counts()
    if dist is not None:
        dist.all_reduce(counts)
    h.update(counts.cpu().numpy().tobytes())
    torch.cuda.synchronize()
    return {"sha256": h.hexdigest(), "trees": K,
            "covers": "feature, threshold and left child of every timed tree; root per-bin row counts "
                      "summed over ranks"}


def run_ours(args):
    import torch
    import torch.distributed as dist
    from yabt_b200 import _lib
    from yabt_b200.boosting import Booster, BoostParams, DeviceData, LogLoss, MSELoss

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # clock sampling runs from here (nvidia-smi takes a moment to start); the
    # summary keeps the samples that fall inside the timed region
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    comm = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        from yabt_b200.distributed import ShardComm
        comm = ShardComm()
    cfg = args.config
    n, F, leaves, depth, loss_name, lr = CONFIGS[cfg]
    # strong scaling: the configuration's n rows are sharded across the ranks in
    # contiguous blocks (the same data set, and so the same model, for every N)
    bounds = [n * r // world for r in range(world + 1)]
    lo, hi = bounds[rank], bounds[rank + 1]
    n_local = hi - lo
    lib = _lib.load()
    X, y = make_data(cfg, n, F, dev, seed=1000)
    if world > 1:
        X, y = X[lo:hi].clone(), y[lo:hi].clone()
        torch.cuda.empty_cache()
    loss = MSELoss() if loss_name == "mse" else LogLoss()
    W, K = args.warmup, args.steps
    P = PHASE_TREES
    params = BoostParams(n_estimators=W + K + P, max_leaves=leaves, max_depth=depth, learning_rate=lr)
    data = DeviceData(X, params.max_bins, dev, comm=comm)
    y_host = y.cpu().numpy()
    del X
    torch.cuda.synchronize()

    ev = {}
    marks = {}

    def cb(t, grower):
        # trees whose deeper levels run in the device-side level loop (a CUDA
        # graph) cannot carry events around each histogram launch; their k_hist
        # time comes from the phase pass instead
        loop = grower.level_loop_start() > 0
        marks["loop"] = loop
        if t == 0 and not loop:
            grower.set_timing(K * grower.levels)      # create the event pool early
        if t == W - 1:
            if not loop:
                grower.set_timing(K * grower.levels)  # restart recording (no allocation)
            grower.acc_reset()
            _lib.check(lib.yabt_launch_count_device_reset(_lib.stream_ptr()), "yabt_launch_count_device_reset")
            ev["start"] = torch.cuda.Event(enable_timing=True)
            ev["start"].record()
            marks["launches0"] = int(lib.yabt_launch_count())
            marks["t0"] = time.time()
        if t == W + K - 1:
            ev["stop"] = torch.cuda.Event(enable_timing=True)
            ev["stop"].record()
            marks["launches1"] = int(lib.yabt_launch_count())
            marks["acc"] = grower.acc_read()          # rows histogrammed by the timed trees (waits for them)
            marks["loop_launches"] = int(lib.yabt_launch_count_device())   # kernels the level loops ran
            if P:
                phases.start()                        # the untimed phase pass: trees W+K .. W+K+P-1

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    from yabt_b200 import phases
    booster = Booster(params, loss)
    booster.fit(None, y_host, data=data, tree_callback=cb, comm=comm)
    torch.cuda.synchronize()
    phase_split = phase_summary(phases, P, dist if world > 1 else None, dev) if P else None
    clocks = sampler.stop((marks["t0"], time.time())) if sampler else None
    ms = ev["start"].elapsed_time(ev["stop"])
    root_rows, child_rows, hist_launches = marks["acc"]
    if marks.get("loop") and phase_split and "hist" in phase_split["ms_per_tree"]:
        hist_ms = [phase_split["ms_per_tree"]["hist"] * K]     # phase pass, per tree, times the timed trees
    else:
        hist_ms = booster.grower_.hist_times()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    trees_per_s = K / (ms / 1000.0)

    # Roofline of the histogram kernel (k_hist): algorithmic bytes of the timed
    # trees = rows histogrammed x (F bin bytes + 4 B gradient [+ 4 B hessian]
    # [+ 4 B row id below the root]); achieved = bytes / summed k_hist time.
    gh = 4 + (4 if loss_name != "mse" else 0)
    alg_bytes = root_rows * (F + gh) + child_rows * (F + gh + 4)
    hist_total_ms = sum(hist_ms)
    achieved = alg_bytes / (hist_total_ms / 1000.0) / 1e9 if hist_total_ms > 0 else float("nan")
    alg_per_launch = alg_bytes / max(hist_launches, 1)
    # DRAM traffic of k_hist per launch: one ncu capture (dram__bytes_read.sum +
    # dram__bytes_write.sum over the k_hist launches of one 2M-row C4 tree) gave
    # 3000.9 MB against 1548.1 MB of algorithmic bytes; scaled by the same
    # algorithmic bytes here (levels below the root read nearly the whole bin
    # matrix, so traffic grows with the rows as the algorithmic bytes do)
    traffic_per_launch = HIST_TRAFFIC_PER_ALG_BYTE * alg_per_launch if cfg == "c4" else None
    avg_hist_ms = hist_total_ms / max(hist_launches, 1)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    # the shared-memory reduction ceiling of k_hist on this GPU (the kernel issues
    # 3 u32 reductions per (row, feature) on the unit-hessian path, 5 otherwise)
    limbs = 3 if loss_name == "mse" else 5
    sink = torch.zeros(1, dtype=torch.int64, device=dev)

    def red_rate(nl: int) -> float:
        pms, pupd = ctypes.c_float(), ctypes.c_longlong()
        best = 0.0
        for _ in range(3):
            _lib.check(lib.yabt_probe_shared_red(nl, 400, sink.data_ptr(), _lib.stream_ptr(), ctypes.byref(pms),
                                                 ctypes.byref(pupd)), "yabt_probe_shared_red")
            best = max(best, pupd.value / (pms.value / 1000.0) / 1e9)
        return best
    red_peak = red_rate(limbs)
    red_peak_root = red_rate(limbs - 1)      # the cached-count root issues one reduction fewer
    red_achieved = (root_rows + child_rows) * F / (hist_total_ms / 1000.0) / 1e9 if hist_total_ms > 0 else 0.0
    # the exact-sum scheme's own ceiling: the timed trees' (row, feature) updates at
    # the measured reduction rates (the root's counts cached after the first tree),
    # i.e. the HBM throughput k_hist would reach with nothing but its reductions
    floor_s = (root_rows * F / (red_peak_root * 1e9) + child_rows * F / (red_peak * 1e9)) if red_peak > 0 else 0.0
    scheme_gbs = alg_bytes / floor_s / 1e9 if floor_s > 0 else float("nan")
    rows_hist = torch.tensor([float(root_rows + child_rows)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(rows_hist)
    bin_reads_per_s = float(rows_hist.item()) * F / (ms / 1000.0)
    digest = model_digest(booster, W, K, dist if world > 1 else None)

    # e2e through the public estimator API from host memory (every rank fits
    # its host shard; the slowest rank's wall time counts)
    e2e = None
    if not args.no_e2e:
        from yabt_b200 import YABTRegressor, YABTClassifier
        del data, booster
        torch.cuda.empty_cache()
        Xh = make_data(cfg, n, F, dev, seed=1000)[0][lo:hi].cpu().pin_memory()
        est_cls = YABTRegressor if loss_name == "mse" else YABTClassifier
        kw = dict(max_leaves=leaves, max_depth=depth, learning_rate=lr)
        # warm-up: one untimed fit of the same data (the analogue of the warm-up
        # steps: context, library, and the allocator's blocks of this size)
        est_cls(n_estimators=1, **kw).fit(Xh, y_host, comm=comm)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        est = est_cls(n_estimators=K, **kw).fit(Xh, y_host, comm=comm)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([dt], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        stages = dict(getattr(est.booster_, "fit_timings_", {}))
        if world > 1 and stages:
            keys = sorted(stages)
            t = torch.tensor([stages[k] for k in keys], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            stages = dict(zip(keys, t.tolist()))
        e2e = {"value": K / dt, "unit": "trees/s",
               "h2d_bytes_per_step": int(n * (F + 1) * 4 / K),   # X and y of every rank, once per fit
               # fit reads back each tree's meta row (4 int32) and leaf-model flag (int32)
               "d2h_bytes_per_step": 4 * 4 + 4,
               "fit_s": dt,
               "warmup": "one untimed fit of the same data and size before the timed fit",
               # host wall seconds of the fit's stages (max over ranks): host->device copy
               # with the transpose, bin fit, bin transform, column moments, then trees
               "stages_s": {k: round(v, 4) for k, v in stages.items()}}
        del Xh, est

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_leg(cfg, dev)

    if rank == 0:
        line = {
            "metric": "trees_per_sec", "value": trees_per_s, "unit": "trees/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded torch Philox, config shapes)",
            "config": workload_config(cfg, world),
            "bin_reads_per_sec": bin_reads_per_s,
            "gpu_launches": marks.get("launches1", 0) - marks.get("launches0", 0) + marks.get("loop_launches", 0),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic_per_launch,
                         "traffic_source": "ncu capture of one 2M-row C4 tree, scaled by algorithmic bytes"
                         if traffic_per_launch else None,
                         "kernel": "k_hist", "alg_bytes_per_launch": alg_per_launch,
                         "avg_launch_ms": avg_hist_ms, "launches_timed": hist_launches,
                         "hist_share_of_step": hist_total_ms / ms,
                         "hist_time_source": "phase pass (the timed trees run their deeper levels in the "
                                             "device-side level loop, which carries no events)"
                         if marks.get("loop") else "CUDA events around each timed k_hist launch",
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650 GB/s"},
            # k_hist is bound by shared-memory reductions, not HBM: its (row, feature)
            # update rate against the same reductions issued alone (yabt_probe_shared_red)
            "atomic_roofline": {"bound": "shared_atomic", "kernel": "k_hist", "achieved": red_achieved,
                                "peak": red_peak, "unit": "G (row, feature) updates/s",
                                "frac": red_achieved / red_peak if red_peak > 0 else None,
                                "u32_reductions_per_update": limbs,
                                # the root level of every tree after the first reuses the fit's
                                # per-bin row counts and issues one reduction fewer per update
                                "root_reductions_per_update_cached_counts": limbs - 1,
                                "peak_root": red_peak_root,
                                "peak_source": "yabt_probe_shared_red, measured in this run",
                                # HBM throughput at that ceiling (algorithmic bytes / time of the
                                # reductions alone) and k_hist's share of it
                                "scheme_ceiling_gbs": scheme_gbs,
                                "scheme_ceiling_frac_of_hbm": scheme_gbs / peak,
                                "achieved_frac_of_scheme_ceiling": achieved / scheme_gbs},
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "model_digest": digest,
            "phases": phase_split,
        }
        print(json.dumps(line))
    if world > 1:
        comm.release_exchange()          # collective: unmap the peers' exchange buffers, free ours
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS))
    ap.add_argument("--ref-rows", type=int, default=2_000_000)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the configuration's row count (small cases for profiling)")
    args = ap.parse_args()
    if args.rows > 0:
        n, *rest = CONFIGS[args.config]
        CONFIGS[args.config] = (args.rows, *rest)
    if args.warmup < 1:
        args.warmup = 1
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "c5":
        run_multiclass(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
