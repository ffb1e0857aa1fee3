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

Beside the timing, every run prints evidence that the timed engine computes
the reference's models: model_sha256 (the e2e model's JSON, identical at every
GPU count in exact mode), parity (at N=1: the engine's model against the
oracle's on the same arrays, JSON bytes and margins bit for bit; for
configs[1] 3 rounds on all 11M rows plus configs[0]'s full 100 rounds),
fast_mode (gpu_math="fast" against exact after 100 rounds) and, for
configs[1], treeshap: configs[4] (TreeSHAP of a 500-tree model of this
workload on 1M fresh rows), rows/s and its largest difference from the
oracle's SHAP values.

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
E2E_RUNS = 3  # e2e runs per bench line; the median is reported
# DRAM bytes / algorithmic bytes of k_hist_stage over one tree: one ncu
# capture of a 4M-row configs[1]-shaped tree (dram__bytes_read.sum +
# dram__bytes_write.sum over its 8 histogram launches); roofline.traffic =
# this ratio x the algorithmic bytes per launch measured live
HIST_TRAFFIC_RATIO = 1800.9 / 8 / 84.44
# oracle rounds compared with the engine's model at N=1 (a few seconds to
# about half a minute of CPU per config)
PARITY_ROUNDS = {"c0": 100, "c1": 3, "c2": 5, "c3": 3, "c3d14": 2, "c1mc": 2}


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


def oracle_train(X, y, params, rounds, feature_types=None, nthread=0):
    """Oracle (C++ restatement of the reference CPU engine) on the workload:
    its model, set-up seconds and per-round wall seconds, `nthread` host
    threads (0 = all)."""
    from oracle import RefCPU
    rc = RefCPU()
    kw = dict(params)
    if feature_types is not None:
        kw["categorical"] = np.array([t == "c" for t in feature_types], np.uint8)
    model = rc.train(X, y, n_rounds=rounds, nthread=nthread, **kw)
    setup, per_round = rc.last_timing()
    return model, setup, per_round


def run_reference(args, rank, world):
    """The reference's CPU engine (the oracle restatement) on the same
    workload: rank 0 alone; W untimed warm-up rounds, then K timed rounds of
    the same training run; `value` = mean timed round x 100, `e2e` = set-up +
    100 x the mean round."""
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    n = args.rows or cfg["rows"]
    X, y, ft = cfg["make"](n)
    t0 = time.perf_counter()
    _, setup, rs = oracle_train(X, y, cfg["params"], args.warmup + args.steps, ft)
    wall = time.perf_counter() - t0
    timed = rs[args.warmup:]
    mean = float(np.mean(timed))
    line = {
        "metric": "train s/100 rounds", "value": round(mean * 100.0, 4), "unit": "s/100 rounds", "n_gpus": world,
        "steps": len(timed), "warmup": args.warmup, "ms_per_step": round(1000 * mean, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": cfg["workload"], "rows": n, "features": int(X.shape[1])},
        "cpu_baseline": {"value": round(mean * 100.0, 4), "unit": "s/100 rounds", "cores": cpu_threads(),
                         "kind": "port",
                         "sample": f"{len(timed)} timed rounds after {args.warmup} warm-up rounds of one training run "
                                   f"on the full {n}-row workload; sketch + quantize set-up {setup:.2f} s; "
                                   f"{wall:.1f} s wall in all"},
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


def _sha256(b):
    import hashlib
    return hashlib.sha256(b).hexdigest()


def _bits_equal(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and bool(np.array_equal(a.view(np.uint32), b.view(np.uint32)))


def parity_vs_oracle(model, oracle_model, X):
    """The engine's model against the oracle's, trained on the same arrays
    with the same parameters: JSON bytes and margins on the training rows,
    bit for bit."""
    ours, ref = model.to_json(), oracle_model.json()
    mo = model.predict(X, output_margin=True)
    mr = oracle_model.predict_margin(X)
    out = {"rounds": int(model.num_trees // max(model.num_outputs, 1)), "rows": int(X.shape[0]),
           "json_equal": ours == ref, "margins_equal": _bits_equal(mo, mr)}
    if not out["margins_equal"]:
        d = np.abs(mo.astype(np.float64) - mr.astype(np.float64))
        out["max_abs_margin_diff"] = float(np.max(d))
        out["rows_differing"] = int(np.count_nonzero(d.reshape(d.shape[0], -1).max(axis=1)))
    if ours != ref:
        k = min(len(ours), len(ref))
        diff = np.nonzero(np.frombuffer(ours[:k], np.uint8) != np.frombuffer(ref[:k], np.uint8))[0]
        out["first_json_difference_at"] = int(diff[0]) if diff.size else k
    return out


def fast_vs_exact(exact, fast, X, y, objective):
    """gpu_math="fast" against the exact model after the same rounds, on the
    training rows: the largest relative prediction error and the loss
    difference (north_star: predictions within 1e-5 relative, logloss within
    1e-4)."""
    a = exact.predict(X, output_margin=True).astype(np.float64)
    b = fast.predict(X, output_margin=True).astype(np.float64)
    if objective == "binary:logistic":
        pa, pb = 1.0 / (1.0 + np.exp(-a)), 1.0 / (1.0 + np.exp(-b))

        def loss(p):
            p = np.clip(p, 1e-15, 1 - 1e-15)
            return float(-np.mean(y * np.log(p) + (1 - y) * np.log(1 - p)))
        name = "logloss"
    elif objective.startswith("multi:"):
        def softmax(m):
            e = np.exp(m - m.max(axis=1, keepdims=True))
            return e / e.sum(axis=1, keepdims=True)
        pa, pb = softmax(a), softmax(b)
        yi = y.astype(np.int64)

        def loss(p):
            return float(-np.mean(np.log(np.clip(p[np.arange(p.shape[0]), yi], 1e-15, 1.0))))
        name = "mlogloss"
    else:
        pa, pb = a, b

        def loss(p):
            return float(np.sqrt(np.mean((p - y) ** 2)))
        name = "rmse"
    rel = (np.abs(pb - pa) / np.maximum(np.abs(pa), 1e-30)).ravel()
    return {"rounds": int(exact.num_trees // max(exact.num_outputs, 1)), "rows": int(X.shape[0]),
            "max_rel_pred_err": float(np.max(rel)), "p99_rel_pred_err": float(np.quantile(rel, 0.99)),
            "median_rel_pred_err": float(np.median(rel)), "preds_over_1e-5": int(np.count_nonzero(rel > 1e-5)),
            f"{name}_exact": loss(pa), f"{name}_fast": loss(pb), f"{name}_diff": abs(loss(pb) - loss(pa)),
            "max_abs_margin_diff": float(np.max(np.abs(b - a)))}


def treeshap_leg(dist, rank, world, device, lib, model, steps, warmup, check_oracle):
    """TreeSHAP and prediction of `model` on 1M fresh N(0,1) rows
    (seed 1), rows sharded over the ranks.  e2e through the public
    Model.predict from host rows; `value` from CUDA events with rows and
    outputs resident.  At N=1 the oracle explains the first 2000 rows with the
    same model (loaded from its JSON): max |SHAP - oracle|, and its rows/s."""
    import torch
    from ferrisboost_b200 import distributed as fbd
    n = 1_000_000
    Xe = np.random.default_rng(1).standard_normal((n, N_FEATURES), dtype=np.float32)
    lo, hi = fbd.shard_range(n, world, rank)
    Xs = np.ascontiguousarray(Xe[lo:hi])
    model.predict(Xs[:1000], pred_contribs=True)
    _fence(dist)
    t0 = time.perf_counter()
    phi = model.predict(Xs, pred_contribs=True)
    e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
    t0 = time.perf_counter()
    margin = model.predict(Xs, output_margin=True)
    pred_e2e_s = _max_over_ranks(dist, time.perf_counter() - t0)
    rowsum_err = float(np.max(np.abs(phi.astype(np.float64).sum(axis=1) - margin.astype(np.float64))))
    xd = torch.from_numpy(Xs).cuda()
    od = torch.empty((hi - lo, N_FEATURES + 1), dtype=torch.float32, device="cuda")
    pd = torch.empty(hi - lo, dtype=torch.float32, device="cuda")
    h = model.device_handle(device)
    s = torch.cuda.current_stream()
    for _ in range(warmup):
        if lib.fbgpu_shap_device(h, xd.data_ptr(), hi - lo, od.data_ptr(), s.cuda_stream):
            raise RuntimeError(lib.fbgpu_last_error(None).decode())
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    l0 = lib.fbgpu_launch_count()
    with ClockSampler(device) as clk:
        _fence(dist)
        ev[0].record(s)
        for _ in range(steps):
            lib.fbgpu_shap_device(h, xd.data_ptr(), hi - lo, od.data_ptr(), s.cuda_stream)
        ev[1].record(s)
        ev[2].record(s)
        for _ in range(steps):
            lib.fbgpu_predict_device(h, xd.data_ptr(), hi - lo, pd.data_ptr(), s.cuda_stream)
        ev[3].record(s)
        _fence(dist)
    launches = lib.fbgpu_launch_count() - l0
    shap_ms = _max_over_ranks(dist, ev[0].elapsed_time(ev[1]) / steps)
    pred_ms = _max_over_ranks(dist, ev[2].elapsed_time(ev[3]) / steps)
    out = {
        "metric": "TreeSHAP rows/s", "value": round(n / (shap_ms / 1000.0), 1), "unit": "rows/s",
        "ms_per_step": round(shap_ms, 3), "steps": steps, "warmup": warmup, "rows": n, "trees": model.num_trees,
        "e2e": {"value": round(n / e2e_s, 1), "unit": "rows/s", "h2d_bytes_per_step": int((hi - lo) * 4 * N_FEATURES),
                "d2h_bytes_per_step": int((hi - lo) * 4 * (N_FEATURES + 1)),
                "includes": "public Model.predict(pred_contribs=True) from host rows"},
        "gpu_launches": int(launches), "clocks": clk.summary(),
        "predict_rows_per_s": round(n / (pred_ms / 1000.0), 1), "predict_e2e_rows_per_s": round(n / pred_e2e_s, 1),
        "max_abs_rowsum_minus_margin": rowsum_err,
        "device_equals_public": bool(np.array_equal(od.cpu().numpy(), phi)),
    }
    del xd, od, pd
    if check_oracle and world == 1:
        from oracle import RefCPU
        doc = model.to_json()
        ref = RefCPU().load_json(doc)
        rows = Xe[:2000]
        ref.shap(rows[:64])
        t0 = time.perf_counter()
        want = ref.shap(rows)
        cpu_s = time.perf_counter() - t0
        out["oracle"] = {"rows": len(rows), "max_abs_err": float(np.max(np.abs(phi[:2000] - want))),
                         "margins_equal": _bits_equal(margin[:2000], ref.predict_margin(rows)),
                         "model_json_round_trip": ref.json() == doc}
        out["cpu_baseline"] = {"value": round(len(rows) / cpu_s, 1), "unit": "rows/s", "cores": cpu_threads(),
                               "kind": "port",
                               "sample": f"oracle TreeSHAP of {len(rows)} of the rows with the same "
                                         f"{model.num_trees}-tree model (loaded from its JSON), all host threads"}
    return out


def atomic_ceiling(lib, device, updates, kernel_ms):
    """The histogram kernels' (row, feature) update rate against the rate the
    same exact update scheme reaches alone (fbgpu_hist_atomic_ceiling: rows
    generated in registers, shared-memory atomics only, every SM), measured
    here on this device."""
    import ctypes as C
    v = C.c_double()
    best = 0.0
    for _ in range(3):
        if lib.fbgpu_hist_atomic_ceiling(device, 0, 8192, C.byref(v)) == 0:
            best = max(best, v.value)
    rate = updates / (kernel_ms / 1000.0)
    return {"unit": "G updates/s", "achieved": round(rate / 1e9, 1), "ceiling": round(best / 1e9, 1),
            "frac": round(rate / best, 4) if best else None,
            "what": "(row, feature) histogram updates per second of the histogram kernels against the same four "
                    "32-bit shared atomics + carry per update with no memory traffic (scheme 0)"}


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
    cpu_legs = rank == 0 and world == 1 and not args.no_cpu

    def train_public(params, rounds, booster=False, data=None):
        Xt, yt = data if data is not None else (X, y)
        if world == 1:
            if booster:
                ds = fb.Dataset(Xt, max_bin=params["max_bin"], feature_types=ft, device=device)
                b = fb.Booster(params, ds, yt)
                b.update(rounds)
                return b
            return fb.train(params, Xt, label=yt, num_boost_round=rounds, feature_types=ft)
        return fbd.train(params, Xt, label=yt, num_boost_round=rounds, feature_types=ft, timeout_s=300,
                         return_booster=booster)

    # untimed: the process's first CUDA work (context creation, module
    # loading) on a few rows, so the e2e leg times the workload, not start-up;
    # when sharded also the process's NCCL communicator, which
    # distributed.train keeps for the process group's later trainings (its
    # start takes from a fraction of a second to seconds, once per process)
    wn = min(n, 4096 * world)
    train_public(p, 2, data=(X[:wn], y[:wn]))

    # e2e: 100 rounds through the public train() from host arrays (sketch,
    # binning, uploads, rounds, model JSON); wall clock, max over ranks; the
    # median of E2E_RUNS runs (the host cores are shared with other jobs, so
    # a single run can catch a stall of the multithreaded set-up), every run
    # listed beside it
    e2e_runs, e2e_split = [], []
    for _ in range(E2E_RUNS):
        _fence(dist)
        t0 = time.perf_counter()
        m = train_public(p, E2E_ROUNDS)
        t1 = time.perf_counter()
        model_json = m.to_json()
        t2 = time.perf_counter()
        e2e_runs.append(_max_over_ranks(dist, t2 - t0))
        e2e_split.append([round(t1 - t0, 4), round(t2 - t1, 4)])
    e2e_s = float(np.median(e2e_runs))
    exact_model = m
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
        same = m.to_json() == model_json.replace(b'"feature_names":[]', b'"feature_names":' + json.dumps(
            names, separators=(",", ":")).encode(), 1)
        del m
        os.remove(path)
        os.rmdir(tmp)
        e2e_parquet = {"value": round(pq_s, 4), "unit": "s/100 rounds", "file_bytes": file_bytes,
                       "model_equals_array_input": same,
                       "includes": "pyarrow decode of the Parquet file + column-major upload + device sketch and "
                                   "binning + 100 rounds + model JSON through the public train(path); wall clock"}

    # device-resident steps: W warm-up rounds, then K rounds timed with CUDA
    # events on the training stream, bracketed by barrier + synchronize.  The
    # timed rounds run as a user's do (no per-level statistics); K more
    # rounds with the statistics on (events and counters around every level)
    # then give the histogram kernels' share, bytes and updates.
    t0 = time.perf_counter()
    b = train_public(p, args.warmup, booster=True)
    setup_s = time.perf_counter() - t0
    fast = train_public(dict(p, gpu_math="fast"), args.warmup, booster=True)
    with ClockSampler(device) as clk:
        _fence(dist)
        l0 = lib.fbgpu_launch_count()
        b.update(args.steps)
        launches = lib.fbgpu_launch_count() - l0
        _fence(dist)
        fast.update(args.steps)
        _fence(dist)
    dev_ms = _max_over_ranks(dist, b.timing()["device_ms"])
    fast_ms = _max_over_ranks(dist, fast.timing()["device_ms"])
    b.set_stats(True)
    _fence(dist)
    b.update(args.steps)
    _fence(dist)
    t = b.timing()
    stats_dev_ms = _max_over_ranks(dist, t["device_ms"])
    comm_ms = _max_over_ranks(dist, t.get("comm_ms", 0.0))
    del fast, b
    ms_step = dev_ms / args.steps
    s100 = ms_step * 100.0 / 1000.0

    hbm_peak, peak_src = _peaks()
    hist_launches = max(t["hist_launches"], 1.0)
    # the histogram kernels alone: the phase's all-reduces (sharded) excluded
    hist_kernel_ms = t["hist_ms"] - t["comm_ms"]
    hist_gbs = t["hist_bytes"] / (hist_kernel_ms / 1000.0) / 1e9 if hist_kernel_ms > 0 else None
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
        "e2e": {"value": round(e2e_s, 4), "unit": "s/100 rounds", "runs": [round(v, 4) for v in e2e_runs],
                "runs_train_json_s": e2e_split,
                "h2d_bytes_per_step": int(e2e_h2d / E2E_ROUNDS),
                "d2h_bytes_per_step": int(tree_readback + 16 + len(model_json) / E2E_ROUNDS),
                "includes": "sketch + binning + upload + 100 rounds + model JSON through the public train(); "
                            "per-rank bytes; wall clock, max over ranks"
                            + ("; the NCCL communicator kept from the untimed warm-up training" if world > 1 else "")},
        **({"e2e_parquet": e2e_parquet} if e2e_parquet else {}),
        "model_sha256": _sha256(model_json),
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(hist_gbs, 1) if hist_gbs else None, "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(hist_gbs / hbm_peak, 4) if hist_gbs else None,
                     "traffic": int(HIST_TRAFFIC_RATIO * t["hist_bytes"] / hist_launches) if hist_gbs else None,
                     "traffic_source": f"ncu dram bytes / algorithmic bytes of one tree at 4M rows (ratio "
                                       f"{HIST_TRAFFIC_RATIO:.2f}), scaled to this launch",
                     "kernel": "k_hist_stage (the histogram kernels of one level), rank 0",
                     "note": None if hist_gbs else "histogram timing is collected on level-wise trees only",
                     "per_launch_ms": round(hist_kernel_ms / hist_launches, 4),
                     "alg_bytes_per_launch": int(t["hist_bytes"] / hist_launches), "peak_source": peak_src},
        "clocks": clk.summary(),
        **({"atomic_ceiling": atomic_ceiling(lib, device, t["hist_updates"], hist_kernel_ms)} if hist_gbs else {}),
        "breakdown": {"hist_share_of_device": round(t["hist_ms"] / t["device_ms"], 4) if t["device_ms"] else None,
                      "stats_rounds_ms_per_round": round(stats_dev_ms / args.steps, 4),
                      "fast_mode_s_per_100_rounds": round(fast_ms / args.steps * 100 / 1000, 4),
                      "setup_s": {"datagen": round(gen_s, 2), "sketch_bin_upload_warmup": round(setup_s, 2)}},
    }
    if world > 1:
        # device ms per round of the per-level histogram all-reduces (the
        # limiting collective), beside the histogram kernels' own ms
        line["breakdown"]["collective_ms_per_round"] = round(comm_ms / args.steps, 4)
        line["breakdown"]["hist_kernel_ms_per_round"] = round(hist_kernel_ms / args.steps, 4)

    # gpu_math="fast" after the same 100 rounds, against the exact model
    objective = p.get("objective", "binary:logistic")
    fast_model = train_public(dict(p, gpu_math="fast"), E2E_ROUNDS)
    if rank == 0:
        line["fast_mode"] = fast_vs_exact(exact_model, fast_model, X, y, objective)
    del fast_model

    # configs[4] rides on the configs[1] run: TreeSHAP of a 500-tree model of
    # this workload (trained through the public train())
    if args.config == "c1" and not args.no_shap:
        trees = 50 if args.rows else 500
        t0 = time.perf_counter()
        shap_model = train_public(p, trees)
        shap_train_s = _max_over_ranks(dist, time.perf_counter() - t0)
        line["treeshap"] = treeshap_leg(dist, rank, world, device, lib, shap_model, steps=min(args.steps, 3),
                                        warmup=1, check_oracle=cpu_legs)
        line["treeshap"]["config"] = {"workload": f"configs[4] TreeSHAP of the {trees}-tree depth-8 configs[1] "
                                                  f"model on 1M N(0,1) rows (seed 1)",
                                      "train_s_for_model": round(shap_train_s, 2)}
        del shap_model

    if cpu_legs:
        # the oracle on the same arrays: its timed rounds are the CPU baseline
        # and its model is compared with the engine's, bit for bit
        R = PARITY_ROUNDS.get(args.config, 3)
        ref, setup, rs = oracle_train(X, y, cfg["params"], R, ft)
        ours = train_public(p, R)
        line["parity"] = {args.config: parity_vs_oracle(ours, ref, X)}
        del ours
        timed = rs[1:] if len(rs) > 1 else rs
        line["cpu_baseline"] = {"value": round(float(np.mean(timed)) * 100, 4), "unit": "s/100 rounds",
                                "cores": cpu_threads(), "kind": "port",
                                "sample": f"{len(timed)} rounds after 1 warm-up round on the full {n}-row workload "
                                          f"(oracle C++ restatement, all host threads); set-up {setup:.2f} s"}
        del ref
        if args.config == "c1" and not args.rows:
            # configs[0] in full: 100 rounds on 1M rows, engine and oracle
            c0 = CONFIGS["c0"]
            X0, y0, _ = c0["make"](c0["rows"])
            p0 = dict(c0["params"], device=f"cuda:{device}")
            ref0, setup0, rs0 = oracle_train(X0, y0, c0["params"], PARITY_ROUNDS["c0"])
            ours0 = train_public(p0, PARITY_ROUNDS["c0"], data=(X0, y0))
            line["parity"]["c0"] = parity_vs_oracle(ours0, ref0, X0)
            line["parity"]["c0"]["oracle_s_per_100_rounds"] = round(float(np.sum(rs0)) * 100 / len(rs0), 4)
            del ours0, ref0
            # the reference CPU engine on one core: 1 warm-up + 2 rounds
            _, setup1, rs1 = oracle_train(X0, y0, c0["params"], 3, nthread=1)
            line["cpu_baseline_1core"] = {"value": round(float(np.mean(rs1[1:])) * 100, 4), "unit": "s/100 rounds",
                                          "cores": 1, "kind": "port", "config": "configs[0]",
                                          "sample": f"2 rounds after 1 warm-up round on configs[0] (1M x 28, depth 6), "
                                                    f"one host thread; set-up {setup1:.2f} s",
                                          "all_cores_value": line["parity"]["c0"]["oracle_s_per_100_rounds"]}
    del exact_model
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
    p = dict(PARAMS, device=f"cuda:{device}")
    t0 = time.perf_counter()
    if world == 1:
        model = fb.train(p, Xtr, label=ytr, num_boost_round=trees)
    else:
        model = fbd.train(p, Xtr, label=ytr, num_boost_round=trees, timeout_s=300)
    train_s = time.perf_counter() - t0
    del Xtr, ytr
    leg = treeshap_leg(dist, rank, world, device, lib, model, args.steps, args.warmup,
                       check_oracle=rank == 0 and world == 1 and not args.no_cpu)
    line = {
        "metric": leg.pop("metric"), "value": leg.pop("value"), "unit": leg.pop("unit"), "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": leg.pop("ms_per_step"), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"configs[4] TreeSHAP of the {trees}-tree depth-8 configs[1] model on 1M N(0,1) "
                               "rows (seed 1)", "rows": leg.pop("rows"), "trees": leg.pop("trees"),
                   "parallelism": f"row shards x{world}"},
        "e2e": leg.pop("e2e"), "gpu_launches": leg.pop("gpu_launches"), "clocks": leg.pop("clocks"),
        **({"cpu_baseline": leg.pop("cpu_baseline")} if "cpu_baseline" in leg else {}),
        **({"oracle": leg.pop("oracle")} if "oracle" in leg else {}),
        "model_sha256": _sha256(model.to_json()),
        "breakdown": dict(leg, train_s_for_model=round(train_s, 2)),
    }
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
    ap.add_argument("--no-shap", action="store_true", help="skip the configs[4] TreeSHAP leg of the configs[1] run")
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
