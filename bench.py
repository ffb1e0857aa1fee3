"""Benchmark: FerrisBoost training on B200, seconds per 100 boosting rounds.

Default workload (the config the metric is quoted
on): 11,000,000 rows x 28 f32 features ~ N(0,1) from seed 0, labels
~ Bernoulli(sigmoid(w.x + 0.5 x0 x1 - 0.3 x2^2)); binary:logistic,
max_bin=256, depthwise max_depth=8, eta=0.1, gpu_math="exact".  A step is one
boosting round over the resident quantized data.  Synthetic data of the
config's shape stands in for HIGGS (not in this container).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config c0|c1|c1mc|c2|c3|c3d14|c4] [--rows R] [--no-cpu] [--parquet]

value: exact-mode s/100 rounds from CUDA events on the training stream, bins
resident in HBM (gradients, glibc-exact expf reproduced on the device,
quantization, the tree's levels and the margin update are all inside the
interval).  e2e: 100 rounds through the public train() from host arrays
(sketch, binning, H2D of the bins and labels, the rounds, model JSON), wall
seconds.  N > 1 (torchrun, one process per GPU): rows are sharded over the
ranks and the library's NCCL communicator all-reduces the per-level
histograms; the total work is fixed (strong scaling) and times are the max
over ranks.  cpu_baseline / --impl reference: the C++ restatement of the
reference CPU engine (oracle/), all host threads, a bounded sample of the same
workload.

--config selects the other benchmark configs (configs[0], [2], [3] and the
max_depth 14 variant of [3], and [4]: TreeSHAP rows/s); they print the same
JSON line for their own workload.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_FEATURES = 28
PARAMS = {"objective": "binary:logistic", "max_depth": 8, "eta": 0.1, "lambda": 1.0, "max_bin": 256}
E2E_ROUNDS = 100
# DRAM bytes / algorithmic bytes of k_hist_stage over one tree, from an ncu
# capture (profiles/k_hist_stage_c1_4Mrows_traffic.md); roofline.traffic =
# this x the algorithmic bytes per launch measured live
HIST_TRAFFIC_RATIO = 1800.9 / 8 / 84.44


def make_data(n, seed=0):
    """configs[0]/[1] generator."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, N_FEATURES), dtype=np.float32)
    w = rng.standard_normal(N_FEATURES)
    z = X @ w + 0.5 * X[:, 0].astype(np.float64) * X[:, 1] - 0.3 * X[:, 2].astype(np.float64) ** 2
    y = (rng.random(n) < 1.0 / (1.0 + np.exp(-z))).astype(np.float32)
    return X, y, None


def make_wide(n, seed=0, F=2000):
    """Uniform(-1, 1) features, labels from 50 random features."""
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1.0, 1.0, (n, F)).astype(np.float32)
    idx = rng.choice(F, 50, replace=False)
    beta = rng.standard_normal(50)
    y = ((X[:, idx] @ beta + rng.normal(0.0, 0.1, n)) > 0).astype(np.float32)
    return X, y, None


def make_mixed(n, seed=0):
    """80 N(0,1) features with 5 % NaN, 20 categorical features
    with 64 codes; target = per-code effects + linear term (NaN as 0) + noise."""
    rng = np.random.default_rng(seed)
    X = np.empty((n, 100), dtype=np.float32)
    X[:, :80] = rng.standard_normal((n, 80), dtype=np.float32)
    codes = rng.integers(0, 64, (n, 20), dtype=np.int32)
    eff = rng.standard_normal((20, 64))
    w = rng.standard_normal(80).astype(np.float32)
    y = (X[:, :80] @ w).astype(np.float64)
    X[:, :80][rng.random((n, 80), dtype=np.float32) < 0.05] = np.nan
    for j in range(20):
        y += eff[j][codes[:, j]]
    X[:, 80:] = codes
    y += rng.normal(0.0, 0.5, n)
    return X, y.astype(np.float32), ["q"] * 80 + ["c"] * 20


def make_multiclass(n, seed=0, K=5):
    """Multiclass workload (none of the benchmark configs is multiclass): configs[1]'s 28
    N(0,1) features; the label is the argmax of K random linear scores plus
    Gumbel noise (a softmax model's draw)."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, N_FEATURES), dtype=np.float32)
    W = rng.standard_normal((N_FEATURES, K)).astype(np.float32) * 0.5
    z = X @ W + rng.gumbel(size=(n, K)).astype(np.float32)
    return X, np.argmax(z, axis=1).astype(np.float32), None


CONFIGS = {
    "c0": dict(make=make_data, rows=1_000_000,
               params=dict(PARAMS, max_depth=6),
               workload="configs[0] binary:logistic 1M x 28, depth 6, max_bin 256, eta 0.1, gpu_math exact"),
    "c1": dict(make=make_data, rows=11_000_000, params=PARAMS,
               workload="configs[1] binary:logistic 11M x 28, depth 8, max_bin 256, eta 0.1, gpu_math exact"),
    "c2": dict(make=make_wide, rows=400_000,
               params=dict(PARAMS, colsample_bytree=0.5),
               workload="configs[2] binary:logistic 400k x 2000 Uniform(-1,1), depth 8, max_bin 256, "
                        "colsample_bytree 0.5, eta 0.1, gpu_math exact"),
    "c3": dict(make=make_mixed, rows=10_000_000,
               params={"objective": "reg:squarederror", "grow_policy": "lossguide", "max_leaves": 255,
                       "max_bin": 1024, "eta": 0.05, "max_depth": 6},
               workload="configs[3] reg:squarederror 10M x (80 numeric, 5% NaN + 20 categorical x 64), "
                        "lossguide max_leaves 255, max_depth 6 (default; the cap does not bind), max_bin 1024, "
                        "eta 0.05, gpu_math exact"),
    "c1mc": dict(make=make_multiclass, rows=11_000_000,
                 params=dict(PARAMS, objective="multi:softprob", num_class=5),
                 workload="multiclass multi:softprob, 5 classes, 11M x 28 (configs[1] shape), depth 8, max_bin 256, "
                          "eta 0.1, gpu_math exact: 5 trees per round"),
    "c3d14": dict(make=make_mixed, rows=10_000_000,
                  params={"objective": "reg:squarederror", "grow_policy": "lossguide", "max_leaves": 255,
                          "max_bin": 1024, "eta": 0.05, "max_depth": 14},
                  workload="configs[3] with max_depth 14: lossguide max_leaves 255 binds (best-first waves), "
                           "10M x 100, max_bin 1024, eta 0.05, gpu_math exact"),
}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device=0):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)  # the first sample lands before the timed work starts
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def cpu_threads():
    return len(os.sched_getaffinity(0))


def reference_rounds(X, y, params, rounds, warmup, feature_types=None):
    """Oracle (C++ restatement of the reference CPU engine) on the workload:
    set-up seconds and per-round wall seconds of the rounds after `warmup`,
    all host threads."""
    from oracle import RefCPU
    rc = RefCPU()
    kw = dict(params)
    if feature_types is not None:
        kw["categorical"] = np.array([t == "c" for t in feature_types], np.uint8)
    rc.train(X, y, n_rounds=warmup + rounds, nthread=0, **kw)
    setup, per_round = rc.last_timing()
    return setup, per_round[warmup:]


def run_reference(args, rank, world):
    """The reference's CPU engine (the oracle restatement) on the same
    workload: rank 0 alone; `value` = mean round x 100, `e2e` = set-up +
    100 rounds."""
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    n = args.rows or cfg["rows"]
    X, y, ft = cfg["make"](n)
    steps = min(args.steps, 10)  # bounded sample: at most 10 timed rounds
    warm = min(args.warmup, 1)
    setup, rs = reference_rounds(X, y, cfg["params"], steps, warm, ft)
    mean = float(np.mean(rs))
    line = {
        "metric": "train s/100 rounds", "value": round(mean * 100.0, 4), "unit": "s/100 rounds", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * mean, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": cfg["workload"].replace(", gpu_math exact", ""), "rows": n,
                   "features": int(X.shape[1])},
        "cpu_baseline": {"value": round(mean * 100.0, 4), "unit": "s/100 rounds", "cores": cpu_threads(),
                         "kind": "port",
                         "sample": f"{steps} timed rounds after {warm} warm-up round(s) on the full {n}-row "
                                   f"workload; sketch + quantize set-up {setup:.2f} s"},
        "e2e": {"value": round(setup + mean * E2E_ROUNDS, 4), "unit": "s/100 rounds", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0, "includes": "set-up + 100 x the mean timed round"},
    }
    print(json.dumps(line), flush=True)


def _dist(world):
    """gloo process group for the barrier and the max over ranks (the training
    collectives are the library's own NCCL communicator)."""
    if world == 1:
        return None
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return dist


def _fence(dist):
    """Barrier + device synchronize, on both sides of a timed region."""
    import torch
    if dist:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(dist, v):
    if not dist:
        return float(v)
    import torch
    t = torch.tensor([float(v)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        peaks = {}
    return float(peaks.get("hbm_gbs", 6650.0)), "measured" if "hbm_gbs" in peaks else "fallback"


def run_ours(args, rank, world):
    import torch
    import ferrisboost_b200 as fb
    from ferrisboost_b200 import distributed as fbd
    from ferrisboost_b200 import _lib
    dist = _dist(world)
    device = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(device)
    lib = _lib.load()
    cfg = CONFIGS[args.config]
    n = args.rows or cfg["rows"]
    t0 = time.perf_counter()
    X, y, ft = cfg["make"](n)
    gen_s = time.perf_counter() - t0
    p = dict(cfg["params"], device=f"cuda:{device}")
    F = int(X.shape[1])
    lo, hi = fbd.shard_range(n, world, rank)

    def train_public(params, rounds, booster=False):
        if world == 1:
            if booster:
                ds = fb.Dataset(X, max_bin=params["max_bin"], feature_types=ft, device=device)
                b = fb.Booster(params, ds, y)
                b.update(rounds)
                return b
            return fb.train(params, X, label=y, num_boost_round=rounds, feature_types=ft)
        return fbd.train(params, X, label=y, num_boost_round=rounds, feature_types=ft, timeout_s=300,
                         return_booster=booster)

    # untimed: the process's first CUDA work (context creation, module
    # loading) on a few rows, so the e2e leg times the workload, not start-up
    wn = min(n, 4096)  # every rank, on its own device: no collectives
    fb.train(p, X[:wn], label=y[:wn], num_boost_round=2, feature_types=ft)

    # e2e: 100 rounds through the public train() from host arrays (sketch,
    # binning, uploads, rounds, model JSON); wall clock, max over ranks
    _fence(dist)
    t0 = time.perf_counter()
    m = train_public(p, E2E_ROUNDS)
    json_bytes = len(m.to_json())
    e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
    ref_json = m.to_json() if args.parquet else None
    del m
    e2e_parquet = None
    if args.parquet and world == 1:
        # the same 100 rounds from a Parquet file of the workload (written
        # untimed): column decode, column-major upload, sketch, binning, rounds
        import tempfile
        import pyarrow as pa
        import pyarrow.parquet as pq
        tmp = tempfile.mkdtemp(prefix="fb_bench_")
        path = os.path.join(tmp, "train.parquet")
        names = [f"f{i}" for i in range(F)]
        pq.write_table(pa.table({**{nm: X[:, i] for i, nm in enumerate(names)}, "label": y}), path,
                       row_group_size=1 << 20)
        file_bytes = os.path.getsize(path)
        t0 = time.perf_counter()
        m = fb.train(p, path, label="label", num_boost_round=E2E_ROUNDS, feature_types=ft)
        pq_s = time.perf_counter() - t0
        same = m.to_json() == ref_json.replace(b'"feature_names":[]', b'"feature_names":' + json.dumps(
            names, separators=(",", ":")).encode(), 1)
        del m
        os.remove(path)
        os.rmdir(tmp)
        e2e_parquet = {"value": round(pq_s, 4), "unit": "s/100 rounds", "file_bytes": file_bytes,
                       "model_equals_array_input": same,
                       "includes": "pyarrow decode of the Parquet file + column-major upload + device sketch and "
                                   "binning + 100 rounds + model JSON through the public train(path); wall clock"}

    # device-resident steps: W warm-up rounds, then K rounds timed with CUDA
    # events on the training stream, bracketed by barrier + synchronize
    t0 = time.perf_counter()
    b = train_public(p, args.warmup, booster=True)
    setup_s = time.perf_counter() - t0
    b.set_stats(True)
    fast = train_public(dict(p, gpu_math="fast"), args.warmup, booster=True)
    with ClockSampler(device) as clk:
        _fence(dist)
        l0 = lib.fbgpu_launch_count()
        b.update(args.steps)
        launches = lib.fbgpu_launch_count() - l0
        _fence(dist)
        fast.update(args.steps)
        _fence(dist)
    t = b.timing()
    dev_ms = _max_over_ranks(dist, t["device_ms"])
    fast_ms = _max_over_ranks(dist, fast.timing()["device_ms"])
    del fast
    ms_step = dev_ms / args.steps
    s100 = ms_step * 100.0 / 1000.0

    hbm_peak, peak_src = _peaks()
    hist_launches = max(t["hist_launches"], 1.0)
    hist_gbs = t["hist_bytes"] / (t["hist_ms"] / 1000.0) / 1e9 if t["hist_ms"] > 0 else None
    rows_local = hi - lo
    depth = p.get("max_depth", 6)
    leaves = p.get("max_leaves", 0) or 2 ** depth
    tree_readback = 32 * min(2 ** (depth + 1), 2 * leaves + 1) + 64
    # host -> device per e2e run: the f32 rows (the device sketches and bins
    # them) and the f32 labels; spread over its 100 rounds
    e2e_h2d = rows_local * (F * 4 + 4)
    line = {
        "metric": "train s/100 rounds", "value": round(s100, 4), "unit": "s/100 rounds", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "config": {"workload": cfg["workload"], "rows": n, "features": F, "parallelism": f"row shards x{world}",
                   "l2": "inputs larger than L2 (bin records and fixed-point gradients exceed 126 MB)"
                   if n * ((F * (2 if p["max_bin"] > 255 else 1) + 15) // 16 * 16 + 16) > 126e6
                   else "inputs smaller than L2"},
        "e2e": {"value": round(e2e_s, 4), "unit": "s/100 rounds",
                "h2d_bytes_per_step": int(e2e_h2d / E2E_ROUNDS),
                "d2h_bytes_per_step": int(tree_readback + 16 + json_bytes / E2E_ROUNDS),
                "includes": "sketch + binning + upload + 100 rounds + model JSON through the public train(); "
                            "per-rank bytes; wall clock, max over ranks"},
        **({"e2e_parquet": e2e_parquet} if e2e_parquet else {}),
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(hist_gbs, 1) if hist_gbs else None, "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(hist_gbs / hbm_peak, 4) if hist_gbs else None,
                     "traffic": int(HIST_TRAFFIC_RATIO * t["hist_bytes"] / hist_launches) if hist_gbs else None,
                     "traffic_source": f"ncu dram bytes / algorithmic bytes of one tree at 4M rows (ratio "
                                       f"{HIST_TRAFFIC_RATIO:.2f}), scaled to this launch",
                     "kernel": "k_hist_stage (the histogram kernels of one level), rank 0",
                     "note": None if hist_gbs else "histogram timing is collected on level-wise trees only",
                     "per_launch_ms": round(t["hist_ms"] / hist_launches, 4),
                     "alg_bytes_per_launch": int(t["hist_bytes"] / hist_launches), "peak_source": peak_src},
        "clocks": clk.summary(),
        "breakdown": {"hist_share_of_device": round(t["hist_ms"] / t["device_ms"], 4) if t["device_ms"] else None,
                      "fast_mode_s_per_100_rounds": round(fast_ms / args.steps * 100 / 1000, 4),
                      "setup_s": {"datagen": round(gen_s, 2), "sketch_bin_upload_warmup": round(setup_s, 2)}},
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        csteps = 2
        setup, rs = reference_rounds(X, y, cfg["params"], csteps, 1, ft)
        line["cpu_baseline"] = {"value": round(float(np.mean(rs)) * 100, 4), "unit": "s/100 rounds",
                                "cores": cpu_threads(), "kind": "port",
                                "sample": f"{csteps} rounds after 1 warm-up round on the full {n}-row workload "
                                          f"(oracle C++ restatement, all host threads)"}
    del b
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_shap(args, rank, world):
    """TreeSHAP and prediction of the 500-tree depth-8 configs[1]
    model on 1M fresh N(0,1) rows (seed 1), rows sharded over the ranks."""
    import torch
    import ferrisboost_b200 as fb
    from ferrisboost_b200 import distributed as fbd
    from ferrisboost_b200 import _lib
    dist = _dist(world)
    device = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(device)
    lib = _lib.load()
    trees = 50 if args.rows else 500
    Xtr, ytr, _ = make_data(args.rows or 11_000_000)
    t0 = time.perf_counter()
    model = fb.train(dict(PARAMS, device=f"cuda:{device}"), Xtr, label=ytr, num_boost_round=trees)
    train_s = time.perf_counter() - t0
    del Xtr, ytr
    n = 1_000_000
    Xe = np.random.default_rng(1).standard_normal((n, N_FEATURES), dtype=np.float32)
    lo, hi = fbd.shard_range(n, world, rank)
    Xs = np.ascontiguousarray(Xe[lo:hi])
    # e2e: public predict(pred_contribs=True) from host rows, results on the host
    model.predict(Xs[:1000], pred_contribs=True)
    _fence(dist)
    t0 = time.perf_counter()
    phi = model.predict(Xs, pred_contribs=True)
    e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
    t0 = time.perf_counter()
    margin = model.predict(Xs, output_margin=True)
    pred_e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
    err = float(np.max(np.abs(phi.astype(np.float64).sum(axis=1) - margin.astype(np.float64))))
    # device-resident: rows and outputs in HBM, CUDA events on the launching stream
    xd = torch.from_numpy(Xs).cuda()
    od = torch.empty((hi - lo, N_FEATURES + 1), dtype=torch.float32, device="cuda")
    pd = torch.empty(hi - lo, dtype=torch.float32, device="cuda")
    h = model.device_handle(device)
    s = torch.cuda.current_stream()
    for _ in range(args.warmup):
        if lib.fbgpu_shap_device(h, xd.data_ptr(), hi - lo, od.data_ptr(), s.cuda_stream):
            raise RuntimeError(lib.fbgpu_last_error(None).decode())
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    l0 = lib.fbgpu_launch_count()
    with ClockSampler(device) as clk:
        _fence(dist)
        ev[0].record(s)
        for _ in range(args.steps):
            lib.fbgpu_shap_device(h, xd.data_ptr(), hi - lo, od.data_ptr(), s.cuda_stream)
        ev[1].record(s)
        ev[2].record(s)
        for _ in range(args.steps):
            lib.fbgpu_predict_device(h, xd.data_ptr(), hi - lo, pd.data_ptr(), s.cuda_stream)
        ev[3].record(s)
        _fence(dist)
    launches = lib.fbgpu_launch_count() - l0
    shap_ms = _max_over_ranks(dist, ev[0].elapsed_time(ev[1]) / args.steps)
    pred_ms = _max_over_ranks(dist, ev[2].elapsed_time(ev[3]) / args.steps)
    same = bool(np.array_equal(od.cpu().numpy(), phi))
    line = {
        "metric": "TreeSHAP rows/s", "value": round(n / (shap_ms / 1000.0), 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(shap_ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"configs[4] TreeSHAP of the {trees}-tree depth-8 configs[1] model on 1M N(0,1) "
                               "rows (seed 1)", "rows": n, "trees": trees, "parallelism": f"row shards x{world}"},
        "e2e": {"value": round(n / e2e_s, 1), "unit": "rows/s",
                "h2d_bytes_per_step": int((hi - lo) * 4 * N_FEATURES),
                "d2h_bytes_per_step": int((hi - lo) * 4 * (N_FEATURES + 1)),
                "includes": "public Model.predict(pred_contribs=True) from host rows"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "breakdown": {"predict_rows_per_s": round(n / (pred_ms / 1000.0), 1),
                      "predict_e2e_rows_per_s": round(n / pred_e2e_s, 1),
                      "max_abs_rowsum_minus_margin": err, "device_equals_public": same,
                      "train_s_for_model": round(train_s, 2)},
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import RefCPU
        rc = RefCPU()
        Xs_tr, ys_tr, _ = make_data(200_000)
        ref = rc.train(Xs_tr, ys_tr, n_rounds=20, nthread=0, **PARAMS)
        rows = Xe[:2000]
        ref.shap(rows[:100])
        t0 = time.perf_counter()
        ref.shap(rows)
        cpu_s = time.perf_counter() - t0
        rps = len(rows) / cpu_s * 20.0 / trees
        line["cpu_baseline"] = {"value": round(rps, 1), "unit": "rows/s", "cores": cpu_threads(), "kind": "port",
                                "sample": f"oracle TreeSHAP of 2000 rows with a 20-tree depth-8 model (200k "
                                          f"training rows), scaled linearly to {trees} trees"}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c1", choices=sorted(CONFIGS) + ["c4"])
    ap.add_argument("--rows", type=int, default=0, help="override the config's row count (smaller runs)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--parquet", action="store_true",
                    help="also time the e2e leg from a Parquet file of the workload (1 GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.gpus > 1 and "WORLD_SIZE" not in os.environ:
        # one process per GPU: relaunch under torchrun on this node
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.gpus}",
               "--master-addr", "127.0.0.1", "--master-port", os.environ.get("MASTER_PORT", "29517"),
               os.path.abspath(__file__)] + sys.argv[1:]
        raise SystemExit(subprocess.call(cmd))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if args.config == "c4":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference arm times training configs; "
                                  "configs[4] TreeSHAP is timed as cpu_baseline of --config c4"}))
            return
        run_reference(args, rank, world)
    elif args.config == "c4":
        run_shap(args, rank, world)
    else:
        run_ours(args, rank, world)


if __name__ == "__main__":
    main()
