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


def _stall_worker(rank, world, port, out_dir):
    """Rank 1 stops taking part between rounds: it stays alive and keeps its
    communicator and memory, but never calls the next round's collectives
    (a stalled host).  Rank 0's next round then waits on its level
    all-reduce until the library's bounded wait (timeout_s) gives up, aborts
    the communicator (which ends the waiting NCCL kernel) and reports the
    timeout; later calls report the failed communicator.  Both ranks leave
    only after rank 0 has seen the error, so no rank's memory goes away
    under a collective."""
    import datetime
    import time
    import torch.distributed as dist
    from ferrisboost_b200 import distributed as fbd
    os.environ["LOCAL_RANK"] = str(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        X, y, _ = _data("logistic_exact")
        b = fbd.train(CASES["logistic_exact"], X, label=y, num_boost_round=2, timeout_s=3,
                      return_booster=True)
        b.model()  # both rounds collected on both ranks
        dist.barrier()
        lines = []
        if rank == 0:
            t0 = time.monotonic()
            try:
                b.update(1)
                b.model()
                lines.append("no error")
            except RuntimeError as e:
                lines.append(f"first {time.monotonic() - t0:.2f} {e}")
            try:
                b.update(1)
                b.model()
                lines.append("no error")
            except RuntimeError as e:
                lines.append(f"second {e}")
        dist.barrier()  # rank 1 waits here, outside any collective, until rank 0 is done
        del b
        fbd.release_communicators()
        with open(os.path.join(out_dir, f"stall_r{rank}.txt"), "w") as f:
            f.write("\n".join(lines))
    finally:
        dist.destroy_process_group()


def test_stalled_peer_ends_in_timeout_then_failed_communicator(tmp_path, monkeypatch):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import time
    import torch.multiprocessing as mp
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")  # plain peer transport, no NVLink multicast objects
    ctx = mp.start_processes(_stall_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 240
    while not ctx.join(timeout=5):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail("ranks did not finish within 240 s")
    lines = (tmp_path / "stall_r0.txt").read_text().splitlines()
    assert (tmp_path / "stall_r1.txt").exists()
    assert lines[0].startswith("first "), lines
    waited = float(lines[0].split()[1])
    assert 2.5 <= waited <= 60.0, lines
    assert "within 3000 ms" in lines[0], lines  # the bounded wait's timeout, not another failure
    assert lines[1].startswith("second ") and "aborted" in lines[1], lines
