"""Host side of row-sharded training, on CPU ranks (gloo, world size 2):
shard ranges, the feature-split sketch (equal to one process's cuts), the
label mean, the NCCL id broadcast and the sharded booster's argument checks.
The device collectives themselves are covered by the 2-GPU test in
test_gpu_distributed.py."""
import ctypes as C
import os
import socket

import numpy as np
import pytest

from ferrisboost_b200 import distributed as fbd


def test_shard_range_covers_rows_in_order():
    for n in (1, 2, 7, 1000, 11_000_001):
        for world in (1, 2, 3, 4, 8):
            if n < world:
                continue
            spans = [fbd.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1
    with pytest.raises(ValueError):
        fbd.shard_range(10, 2, 2)


def test_label_mean_matches_sequential_f64():
    from ferrisboost_b200 import lib, _lib
    rng = np.random.default_rng(3)
    y = (rng.random(10001) < 0.3).astype(np.float32)
    w = rng.random(10001).astype(np.float32)
    acc = 0.0
    for v in y:
        acc = acc + float(v) / len(y)
    got = lib().fb_label_mean(_lib.ptr(y, C.c_float), None, len(y))
    assert np.float32(got) == np.float32(acc)
    sw = 0.0
    for v in w:
        sw = sw + float(v)
    acc = 0.0
    for a, b in zip(y, w):
        acc = acc + float(a) / sw * float(b)
    got = lib().fb_label_mean(_lib.ptr(y, C.c_float), _lib.ptr(w, C.c_float), len(y))
    assert np.float32(got) == np.float32(acc)


def test_sketch_features_equal_dataset_cuts():
    import ferrisboost_b200 as fb
    rng = np.random.default_rng(5)
    X = rng.standard_normal((20000, 6)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    X[:, 4] = rng.integers(0, 9, 20000)
    ft = ["q", "q", "q", "q", "c", "q"]
    ds = fb.Dataset(X, max_bin=64, feature_types=ft)
    cuts, off = ds.cuts()
    got = fbd.sketch_features(X, [5, 0, 4], 64, categorical=np.array([0, 0, 0, 0, 1, 0], np.uint8))
    for f, c in zip([5, 0, 4], got):
        assert np.array_equal(c, cuts[off[f]:off[f + 1]])
    # a dataset binned from given cuts equals the sketched one, shard by shard
    lo, hi = 7000, 20000
    part = fb.Dataset(X[lo:hi], max_bin=64, feature_types=ft, cuts=(cuts, off))
    for f in range(6):
        assert np.array_equal(part.column(f), ds.column(f)[lo:hi])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    import ferrisboost_b200 as fb
    from ferrisboost_b200 import distributed as fbd
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        X = rng.standard_normal((30000, 9)).astype(np.float32)
        X[rng.random(X.shape) < 0.02] = np.nan
        cuts, off = fbd.sketch_cuts(X, 128)
        # the NCCL id travels from rank 0 unchanged (ids are random bytes; no GPU needed to make one)
        nid = fbd._broadcast(os.urandom(128) if rank == 0 else None)
        ids = [None] * world
        dist.all_gather_object(ids, nid)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), cuts=cuts, off=off, same_id=all(i == ids[0] for i in ids))
        # a sharded booster without base_score is refused before any device work
        lo, hi = fbd.shard_range(len(X), world, rank)
        ds = fb.Dataset(X[lo:hi], max_bin=128, cuts=(cuts, off))
        y = np.zeros(hi - lo, np.float32)
        err = ""
        try:
            fb.Booster({"objective": "binary:logistic"}, ds, y,
                       shard=fb.Shard(lo, len(X), nid, world, rank, float("nan")))
        except ValueError as e:
            err = str(e)
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(err)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_share_cuts_and_id(tmp_path):
    import torch.multiprocessing as mp
    import ferrisboost_b200 as fb
    world, port = 2, _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    rng = np.random.default_rng(11)
    X = rng.standard_normal((30000, 9)).astype(np.float32)
    X[rng.random(X.shape) < 0.02] = np.nan
    want_cuts, want_off = fb.Dataset(X, max_bin=128).cuts()
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        assert np.array_equal(z["cuts"], want_cuts) and np.array_equal(z["off"], want_off)
        assert bool(z["same_id"])
        assert "base_score" in (tmp_path / f"err{r}.txt").read_text()


def _liveness_worker(rank, world, port, out_dir, scenario):
    import datetime
    import time
    import torch.distributed as dist
    from ferrisboost_b200.distributed import Liveness, PeerLost
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    live = Liveness(store, rank, world, stale_s=2.0, prefix=scenario)
    outcome = "ok"
    try:
        for step in range(6):
            if rank == 1 and step == 3:
                if scenario == "leave":
                    live.leave()  # a graceful early exit between rounds
                break             # "stall": stop beating without a word
            live.beat()
            if step == 4:
                time.sleep(2.5)   # past stale_s: a stalled peer is now stale
            live.check()
            time.sleep(0.2)
    except PeerLost as e:
        outcome = f"lost: {e}"
    with open(os.path.join(out_dir, f"{scenario}{rank}.txt"), "w") as f:
        f.write(outcome)
    if rank == 0:
        time.sleep(0.5)  # keep the store's server up until rank 1 is done with it


@pytest.mark.parametrize("scenario", ["leave", "stall"])
def test_liveness_detects_a_lost_peer_before_the_next_round(tmp_path, scenario):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_liveness_worker, args=(2, port, str(tmp_path), scenario), nprocs=2, join=True,
                       start_method="spawn")
    r0 = (tmp_path / f"{scenario}0.txt").read_text()
    assert r0.startswith("lost: rank 1"), r0
    if scenario == "leave":
        assert "left" in r0
    else:
        assert "has not answered" in r0


class _FakeComm:
    """Stands in for distributed.Communicator: no NCCL, no GPU."""

    def __init__(self, nid, world, rank, device, timeout_ms):
        self.nid, self.timeout_ms, self.held, self.aborted = bytes(nid), timeout_ms, False, False

    def usable(self):
        return not self.held and not self.aborted

    def abort(self):
        self.aborted = True


def _comm_cache_worker(rank, world, port, out_dir):
    import json
    import torch.distributed as dist
    from ferrisboost_b200 import distributed as fbd
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    fbd.Communicator = _FakeComm
    fbd.nccl_unique_id = lambda: os.urandom(128)
    try:
        key = (0, world, rank, 0)
        first = fbd._communicator(key, world, rank, 0, 5000)
        again = fbd._communicator(key, world, rank, 0, 5000)  # every rank holds the same usable one
        if rank == 1:
            again.held = True  # a live booster still holds rank 1's communicator
        third = fbd._communicator(key, world, rank, 0, 5000)
        other_timeout = fbd._communicator(key, world, rank, 0, 9000)
        ids = [None] * world
        dist.all_gather_object(ids, (first.nid, third.nid, other_timeout.nid))
        res = {"reused": again is first, "replaced": third is not again,
               "first_aborted": first.aborted, "third_aborted": third.aborted,
               "same_ids": all(i == ids[0] for i in ids),
               "new_on_timeout": other_timeout is not third, "kept": len(fbd._COMMS)}
        fbd.release_communicators()
        res["released"] = other_timeout.aborted and not fbd._COMMS
        with open(os.path.join(out_dir, f"c{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


def test_communicator_kept_between_trainings_only_when_every_rank_can_use_it(tmp_path):
    import json
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    mp.start_processes(_comm_cache_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r0 = json.loads((tmp_path / "c0.json").read_text())
    r1 = json.loads((tmp_path / "c1.json").read_text())
    for r in (r0, r1):
        assert r["reused"] and r["replaced"] and r["same_ids"] and r["new_on_timeout"]
        assert r["kept"] == 1 and r["released"] and not r["third_aborted"]
    # rank 0 could use its copy but rank 1 could not: rank 0 ends it without waiting
    # for rank 1; rank 1's copy stays with the booster that holds it
    assert r0["first_aborted"] and not r1["first_aborted"]
