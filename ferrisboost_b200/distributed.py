"""Row-sharded training on the GPUs of one node, one process per GPU.

Each rank holds a contiguous range of the rows (``shard_range``).  The ranks
split the per-feature quantile sketch between them and exchange the cuts, bin
only their own rows, and grow every tree together: the library runs NCCL
collectives on its training stream for the gradient bounds and root sum of
each round and for the accumulated node histograms and per-node row counts of
each level.  The histograms are sums of integers modulo 2^64, so in exact mode
every rank ends with the model a single GPU trains on all the rows, byte for
byte.

The reference trains on one GPU only; its communication trait has a
single-process ``Local`` implementation (src/training/comm.rs:10-41).  This
module is the multi-GPU replacement for that trait.

    torchrun --nproc-per-node 8 my_train.py   # in my_train.py:
    torch.distributed.init_process_group("gloo")
    model = ferrisboost_b200.distributed.train(params, X, label=y, num_boost_round=100)

``torch.distributed`` (any backend; gloo is enough) only carries the NCCL id,
the cuts and the label mean between the ranks before training.

The NCCL communicator is made by the first ``train`` of a process group and
kept for the next ones (starting one takes from a fraction of a second to
seconds, like the process group itself); ``release_communicators`` ends the
kept ones.
"""
from __future__ import annotations

import atexit
import ctypes as C
import hashlib
import os
import sys
from typing import Any, Mapping, Sequence

import numpy as np

from . import (_OBJECTIVES, Booster, Dataset, Shard, _as_matrix, _err, _feature_flags, _lib, _normalize_params,
               lib)
from ._trace import PhaseTrace

__all__ = ["shard_range", "sketch_cuts", "nccl_unique_id", "train", "Liveness", "PeerLost", "Communicator",
           "release_communicators"]


class Communicator:
    """An NCCL communicator started before the data is prepared
    (fbgpu_comm_begin): its initialization and a warm-up of the collectives
    run on a background thread of the library while this rank sketches and
    bins its rows.  Every rank creates one with the same unique id; a
    Booster built with ``Shard(comm=...)`` shares it; the communicator ends
    when this object and every booster holding it are gone."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int, timeout_ms: int = 120000):
        nid = np.frombuffer(unique_id, dtype=np.uint8).copy()
        h = C.c_void_p()
        st = lib().fbgpu_comm_begin(_lib.ptr(nid, C.c_uint8), nranks, rank, device, timeout_ms, C.byref(h))
        if st:
            raise RuntimeError(lib().fbgpu_last_error(None).decode())
        self.handle = h
        self.timeout_ms = timeout_ms

    def usable(self) -> bool:
        """Started without error, not failed, and held by no live booster."""
        return bool(self.handle) and lib().fbgpu_comm_usable(self.handle) == 1

    def abort(self) -> None:
        """Ends the communicator without waiting for the peers (nothing may be
        in flight on it)."""
        if self.handle:
            lib().fbgpu_comm_abort(self.handle)

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                lib().fbgpu_comm_free(h)
            except TypeError:  # interpreter shutdown: module globals already cleared
                pass
            self.handle = None


# Communicators kept between trainings: (group, world, rank, device) ->
# (Communicator, generation).  The generation names the unique id the
# communicator was made from, the same on every rank that made it together.
_COMMS: dict = {}


def release_communicators() -> None:
    """Ends every communicator this process keeps (at exit too).  Call it on
    every rank; boosters still holding one fail their next collective."""
    while _COMMS:
        _, (comm, _gen) = _COMMS.popitem()
        comm.abort()
        del comm


atexit.register(release_communicators)


def _all_gather(obj, group=None) -> list:
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


def _communicator(key, world: int, rank: int, device: int, timeout_ms: int, group=None):
    """The kept communicator of ``key`` when every rank holds the same usable
    one, else a new one from a unique id of rank 0 (kept for the next
    training).  Every rank takes the same branch: one all-gather of the kept
    generations decides, before any NCCL call."""
    kept = _COMMS.get(key)
    mine = kept[1] if kept is not None and kept[0].timeout_ms == timeout_ms and kept[0].usable() else None
    gens = _all_gather(mine, group)
    if mine is not None and all(g == mine for g in gens):
        return kept[0]
    if kept is not None:
        del _COMMS[key]
        if mine is not None:  # a peer cannot use it: end it here without waiting for that peer
            kept[0].abort()
        del kept
    nid = None
    if rank == 0:  # a failure on rank 0 is sent to every rank, which all raise
        try:
            nid = nccl_unique_id()
        except RuntimeError as e:
            nid = "error: " + str(e)
    nid = _broadcast(nid, group)
    if isinstance(nid, str):
        raise RuntimeError(f"rank 0 could not create an NCCL id ({nid})")
    comm = Communicator(nid, world, rank, device, timeout_ms)
    _COMMS[key] = (comm, hashlib.blake2b(nid, digest_size=8).hexdigest())
    return comm


class PeerLost(RuntimeError):
    """A rank of the run left or stopped answering; raised on the host before
    any collective is launched, so no GPU waits on the missing rank."""


class Liveness:
    """Host-side liveness of the ranks through the process group's key-value
    store.  Every rank stamps a heartbeat before each round; a rank that ends
    early marks itself as left.  ``check()`` raises PeerLost when a peer has
    left or its heartbeat is older than ``stale_s``, so the surviving ranks stop
    between rounds instead of entering a collective that cannot complete.  The
    library's bounded NCCL waits (``timeout_s`` of ``train``) remain the last
    resort for a rank that dies inside a round."""

    def __init__(self, store, rank: int, world: int, stale_s: float = 60.0, prefix: str = "fbgpu"):
        import datetime
        self.store, self.rank, self.world, self.stale_s, self.prefix = store, rank, world, stale_s, prefix
        self.beat()
        # every rank's first heartbeat, within stale_s
        for r in range(world):
            try:
                store.wait([self._key("beat", r)], datetime.timedelta(seconds=stale_s))
            except Exception as e:  # the store's timeout error
                raise PeerLost(f"rank {r} never joined the run") from e

    def _key(self, kind: str, r: int) -> str:
        return f"{self.prefix}/{kind}/{r}"

    def beat(self) -> None:
        import time
        self.store.set(self._key("beat", self.rank), repr(time.time()))

    def leave(self) -> None:
        self.store.set(self._key("left", self.rank), "1")

    def check(self) -> None:
        import time
        now = time.time()
        for r in range(self.world):
            if r == self.rank:
                continue
            if self.store.check([self._key("left", r)]):
                raise PeerLost(f"rank {r} left the run")
            if not self.store.check([self._key("beat", r)]):
                raise PeerLost(f"rank {r} never joined the run")
            age = now - float(self.store.get(self._key("beat", r)).decode())
            if age > self.stale_s:
                raise PeerLost(f"rank {r} has not answered for {age:.1f} s")


def shard_range(n_rows: int, world_size: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of ``rank``: contiguous, sizes differing by at most one."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"invalid rank {rank} of world size {world_size}")
    base, extra = divmod(int(n_rows), world_size)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (made on rank 0, sent to the others)."""
    buf = np.zeros(128, dtype=np.uint8)
    st = lib().fbgpu_nccl_unique_id(_lib.ptr(buf, C.c_uint8))
    if st:
        raise RuntimeError(lib().fbgpu_last_error(None).decode())
    return buf.tobytes()


def sketch_features(X: np.ndarray, feats: Sequence[int], max_bin: int, weight=None, categorical=None,
                    nthread: int = 0, device: int | None = None) -> list[np.ndarray]:
    """Cuts of the listed features (the sketch of ``Dataset``, feature by
    feature); on CUDA device ``device`` when given (the same cuts)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    fs = np.ascontiguousarray(feats, dtype=np.uint32)
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    cat = None if categorical is None else np.ascontiguousarray(categorical, dtype=np.uint8)
    cap = sum(65534 if cat is not None and cat[f] else max(max_bin, 1) for f in fs) + 1
    cuts = np.zeros(cap, dtype=np.float32)
    counts = np.zeros(max(len(fs), 1), dtype=np.uint32)
    if device is None:
        n = lib().fb_sketch_features(_lib.ptr(X, C.c_float), X.shape[0], X.shape[1], max_bin, _lib.ptr(w, C.c_float),
                                     _lib.ptr(cat, C.c_uint8), _lib.ptr(fs, C.c_uint32), len(fs), nthread,
                                     _lib.ptr(cuts, C.c_float), _lib.ptr(counts, C.c_uint32), cap)
    else:
        n = lib().fb_sketch_features_device(_lib.ptr(X, C.c_float), X.shape[0], X.shape[1], max_bin,
                                            _lib.ptr(w, C.c_float), _lib.ptr(cat, C.c_uint8), _lib.ptr(fs, C.c_uint32),
                                            len(fs), nthread, int(device), _lib.ptr(cuts, C.c_float),
                                            _lib.ptr(counts, C.c_uint32), cap)
    if n < 0:
        raise ValueError(_err())
    out, at = [], 0
    for i in range(len(fs)):
        out.append(cuts[at:at + counts[i]].copy())
        at += int(counts[i])
    return out


def sketch_cuts(X: np.ndarray, max_bin: int, weight=None, categorical=None, nthread: int = 0, group=None,
                device: int | None = None):
    """(cut values, F+1 offsets) of all rows of X, the features sketched
    round-robin by the ranks of ``group`` (each on its CUDA device when
    ``device`` is given) and all-gathered.  Equal to the cuts one process
    sketches alone."""
    import torch.distributed as dist
    F = X.shape[1]
    rank, world = _rank_world(group)
    mine = list(range(rank, F, world))
    local = sketch_features(X, mine, max_bin, weight, categorical, nthread, device)
    gathered: list = [None] * world
    if world > 1:
        dist.all_gather_object(gathered, (mine, [c.tobytes() for c in local]), group=group)
    else:
        gathered = [(mine, [c.tobytes() for c in local])]
    per = [None] * F
    for feats, cuts in gathered:
        for f, c in zip(feats, cuts):
            per[f] = np.frombuffer(c, dtype=np.float32)
    off = np.zeros(F + 1, dtype=np.uint32)
    off[1:] = np.cumsum([len(c) for c in per])
    vals = np.concatenate(per) if off[-1] else np.zeros(0, np.float32)
    return vals.astype(np.float32), off


def _rank_world(group=None) -> tuple[int, int]:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def _broadcast(obj, group=None):
    import torch.distributed as dist
    box = [obj]
    dist.broadcast_object_list(box, src=0, group=group)
    return box[0]


def train(params: Mapping[str, Any], data: Any, label: Any = None, num_boost_round: int = 10, weight: Any = None,
          feature_types: Sequence[str] | None = None, group=None, timeout_s: float = 120.0,
          return_booster: bool = False, liveness: Liveness | None = None):
    """``ferrisboost_b200.train`` over all ranks of ``group`` (an initialised
    ``torch.distributed`` process group; one process per GPU).

    Every rank passes the whole data set (as each reads the same file); rank
    r bins and trains rows ``shard_range(n, world, r)`` on ``cuda:LOCAL_RANK``
    (unless ``params["device"]`` names one).  Returns the model, identical on
    every rank (or the booster with ``return_booster``).  Collective waits
    give up after ``timeout_s`` with a RuntimeError on the ranks still waiting.
    With ``liveness``, the rounds run one at a time and every rank checks its
    peers before each round (PeerLost).
    """
    rank, world = _rank_world(group)
    params = dict(params)
    if params.get("device") in (None, "cuda", "gpu"):
        params["device"] = f"cuda:{int(os.environ.get('LOCAL_RANK', rank))}"
    if not params.get("nthread"):
        local = int(os.environ.get("LOCAL_WORLD_SIZE", world))
        params["nthread"] = max(1, len(os.sched_getaffinity(0)) // max(local, 1))
    p = _normalize_params(params, num_boost_round)
    if label is None:
        raise ValueError("label is required for array input")
    X = _as_matrix(data, p["missing"])
    n, F = X.shape
    y = np.ascontiguousarray(label, dtype=np.float32)
    if y.shape != (n,):
        raise ValueError(f"label has shape {y.shape}, expected ({n},)")
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    if world == 1:
        from . import train as train_one
        return train_one(params, X, label=y, num_boost_round=num_boost_round, weight=w, feature_types=feature_types)
    if n < world:  # the same on every rank: all raise before any collective
        raise ValueError(f"{n} rows cannot be sharded over {world} ranks")
    cat = _feature_flags(feature_types, F)
    trace = PhaseTrace(f"rank {rank}")
    timeout_ms = int(max(1.0, timeout_s) * 1000)
    # a new communicator initializes while the cuts are sketched and the rows binned
    comm = _communicator((id(group) if group is not None else 0, world, rank, p["device_index"]), world, rank,
                         p["device_index"], timeout_ms, group)
    trace("id, communicator start")
    cuts = sketch_cuts(X, p["max_bin"], w, cat, p["nthread"], group, device=p["device_index"])
    trace("sketch + all-gather of cuts")
    lo, hi = shard_range(n, world, rank)
    base = p["base_score"]
    class_margins = None
    if p["objective"].startswith("multi:"):
        # every rank holds all labels: the class base margins over all rows
        if base is None:
            class_margins = np.zeros(p["num_class"], np.float32)
            if lib().fb_class_margins(_lib.ptr(y, C.c_float), _lib.ptr(w, C.c_float), n, p["num_class"],
                                      _lib.ptr(class_margins, C.c_float)):
                raise ValueError((lib().fb_last_error() or b"").decode())
            base = float("nan")
    elif base is None:  # over all rows, as a single process would (objective.rs:403-493)
        base = float(lib().fb_initial_base_score(_OBJECTIVES[p["objective"]], _lib.ptr(y, C.c_float),
                                                 _lib.ptr(w, C.c_float), n, p["scale_pos_weight"]))
    trace("base score")
    ds = Dataset(X[lo:hi], max_bin=p["max_bin"], feature_types=feature_types, nthread=p["nthread"], cuts=cuts,
                 device=p["device_index"])
    trace("shard binning")
    shard = Shard(row_offset=lo, n_rows_global=n, nccl_id=b"", nranks=world, rank=rank, base_score=base,
                  timeout_ms=timeout_ms, comm=comm, class_margins=class_margins)
    b = Booster(params, ds, y[lo:hi], None if w is None else w[lo:hi], shard=shard)
    trace("booster (communicator ready)")
    if liveness is None:
        b.update(num_boost_round)
        trace("rounds")
    else:
        for _ in range(num_boost_round):
            liveness.beat()
            liveness.check()
            b.update(1)
    if return_booster:
        return b
    m = b.model()
    m.params = p
    return m
