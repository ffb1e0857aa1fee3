"""Row-sharded training on 2 GPUs (one process per GPU, NCCL collectives on
the training stream): every rank's model equals the single-GPU model byte for
byte, in exact and in fast mode, with row and column sampling, categorical
features (one of 1,000 codes), a multiclass objective and best-first
lossguide, both with the feature-sharded split search (reduce-scatter of the
level histograms, gather of the per-node winners; FBGPU_SPLIT_SHARD=1) and
with the all-reduce of every bin (FBGPU_SPLIT_SHARD=0).  Needs at least 2
GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = {
    "logistic_exact": {"objective": "binary:logistic", "max_depth": 6, "eta": 0.3, "max_bin": 64},
    "sampled_categorical": {"objective": "binary:logistic", "max_depth": 5, "eta": 0.2, "max_bin": 300,
                            "subsample": 0.8, "colsample_bytree": 0.7, "seed": 7},
    "sqerr_fast": {"objective": "reg:squarederror", "max_depth": 7, "eta": 0.1, "gpu_math": "fast"},
    "multiclass": {"objective": "multi:softprob", "num_class": 4, "max_depth": 5, "eta": 0.3, "max_bin": 128,
                   "subsample": 0.9, "seed": 3},
    "wide_categorical": {"objective": "reg:squarederror", "max_depth": 6, "eta": 0.3, "max_bin": 64},
    "lossguide_cap": {"objective": "binary:logistic", "grow_policy": "lossguide", "max_leaves": 10, "max_depth": 8,
                      "eta": 0.3, "max_bin": 64},
}


def _data(case):
    rng = np.random.default_rng(21)
    n, F = 150_001, 10
    X = rng.standard_normal((n, F)).astype(np.float32)
    X[rng.random(X.shape) < 0.03] = np.nan
    ft = None
    if case == "sampled_categorical":
        X[:, 3] = rng.integers(0, 12, n)
        ft = ["q"] * F
        ft[3] = "c"
    if case == "wide_categorical":
        X[:, 8] = rng.integers(0, 1000, n)
        X[:, 8][rng.random(n) < 0.02] = np.nan
        ft = ["q"] * F
        ft[8] = "c"
    z = X[:, 0] + 0.5 * np.nan_to_num(X[:, 1]) * np.nan_to_num(X[:, 2])
    if case == "wide_categorical":
        z = z + np.sin(np.nan_to_num(X[:, 8]))
    if CASES[case]["objective"] == "binary:logistic":
        y = (rng.random(n) < 1 / (1 + np.exp(-np.nan_to_num(z)))).astype(np.float32)
    elif CASES[case]["objective"].startswith("multi:"):
        y = np.digitize(np.nan_to_num(z), [-1.0, 0.0, 1.0]).astype(np.float32)
    else:
        y = np.nan_to_num(z).astype(np.float32)
    return X, y, ft


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, split_shard):
    import datetime
    import torch.distributed as dist
    from ferrisboost_b200 import distributed as fbd
    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["FBGPU_SPLIT_SHARD"] = split_shard
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        gens = []
        for case, params in CASES.items():
            X, y, ft = _data(case)
            m = fbd.train(params, X, label=y, num_boost_round=6, feature_types=ft, timeout_s=60)
            with open(os.path.join(out_dir, f"{case}_r{rank}.json"), "wb") as f:
                f.write(m.to_json())
            gens += [g for _, g in fbd._COMMS.values()]
        # one communicator, made by the first training and kept for the others
        with open(os.path.join(out_dir, f"gens_r{rank}.txt"), "w") as f:
            f.write(" ".join(gens))
        fbd.release_communicators()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split_shard", ["1", "0"])
def test_two_gpu_models_equal_single_gpu(tmp_path, split_shard):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import ferrisboost_b200 as fb
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), split_shard), nprocs=world, join=True,
                       start_method="spawn")
    for case, params in CASES.items():
        X, y, ft = _data(case)
        want = fb.train(dict(params, device="cuda:0"), X, label=y, num_boost_round=6, feature_types=ft).to_json()
        for r in range(world):
            got = (tmp_path / f"{case}_r{r}.json").read_bytes()
            assert got == want, f"{case}: rank {r} model differs from the single-GPU model"
    gens = [(tmp_path / f"gens_r{r}.txt").read_text().split() for r in range(world)]
    assert len(gens[0]) == len(CASES) and len(set(gens[0])) == 1 and gens[0] == gens[1]
