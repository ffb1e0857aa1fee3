"""ferrisboost_b200 — FerrisBoost's training and explanation engine on B200.

Drop-in for the reference's Python entry points (python/ferrisboost/__init__.py
of mdai001/FerrisBoost): ``train(params, data, label=..., num_boost_round=...)``
returns a ``Model`` with ``predict(..., output_margin, pred_contribs)``,
``save_model`` and the XGBoost-compatible JSON.  Parameters use the
reference's names, aliases and defaults; unknown names raise ``ValueError``.

Every training, prediction and SHAP call runs on a CUDA device through the
in-tree library libfbgpu.so (C ABI in include/fbgpu.h and include/fb_engine.h):
there is no CPU execution path, and a missing library or device raises.
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os
from typing import Any, Mapping, NamedTuple, Sequence

import numpy as np

from . import _lib, columnar

__all__ = ["train", "Model", "Booster", "Dataset", "build", "lib"]

_DEFAULTS: dict[str, Any] = {  # python/ferrisboost/__init__.py:47-157 (the subset this engine runs)
    "objective": "binary:logistic",
    "max_depth": 6,
    "max_leaves": 0,
    "grow_policy": "depthwise",
    "max_bin": 255,
    "eta": 0.3,
    "lambda": 1.0,
    "gamma": 0.0,
    "alpha": 0.0,
    "max_delta_step": None,
    "scale_pos_weight": 1.0,
    "min_child_weight": 1.0,
    "subsample": 1.0,
    "sampling_method": "uniform",
    "colsample_bytree": 1.0,
    "colsample_bylevel": 1.0,
    "colsample_bynode": 1.0,
    "cols_per_block": None,
    "nthread": 0,
    "hist_streams": None,
    "resident_blocks": None,
    "hist_nodes_per_batch": None,
    "gpu_math": None,
    "device": None,
    "gpu_memory_budget": None,
    "device_quantize": None,
    "seed": 0,
    "base_score": None,
    "monotone_constraints": None,
    "enable_categorical": False,
    "missing": float("nan"),
    "max_cat_to_onehot": 4,
    "max_cat_threshold": 64,
    "num_class": 0,
}
_ALIASES = {  # python/ferrisboost/__init__.py:160-167
    "learning_rate": "eta",
    "reg_lambda": "lambda",
    "reg_alpha": "alpha",
    "n_jobs": "nthread",
    "random_state": "seed",
}
# Accepted for drop-in compatibility; the device planner owns these choices
# (every configuration is resident in HBM), so their values do not change the model.
_PLANNER_OWNED = ("cols_per_block", "hist_streams", "resident_blocks", "hist_nodes_per_batch", "gpu_memory_budget",
                  "device_quantize")
_OBJECTIVES = {"reg:squarederror": 0, "binary:logistic": 1, "multi:softprob": 2, "multi:softmax": 3}


def lib():
    return _lib.load()


def build(force: bool = False):
    """Compile libfbgpu.so in-tree (nvcc, sm_100a)."""
    from .build import build as _build
    return _build(force=force)


def _int_param(name: str, raw: Any) -> int:
    """XGBoost writes every parameter as a string (tree.rs:1082-1095 parse_param)."""
    try:
        return int(str(raw).strip())
    except ValueError:
        raise ValueError(f"{name} = {raw!r} is not an integer") from None


def _base_scores(raw: Any, multi: bool) -> list:
    """tree.rs:1034-1080: "5E-1" (1.x / 2.x) or "[5E-1]" (3.x); a vector
    "[a,b,c]" only for multiclass models."""
    t = str(raw).strip()
    inner = t[1:-1] if t.startswith("[") and t.endswith("]") else t
    parts = [p.strip() for p in inner.split(",") if p.strip()]
    if not parts:
        raise ValueError(f"base_score is empty: {raw!r}")
    if len(parts) > 1 and not multi:
        raise ValueError(f"base_score is a vector ({raw!r}); multi-target models are not supported")
    try:
        return [np.float32(float(p)) for p in parts]
    except ValueError:
        raise ValueError(f"base_score = {raw!r} is not a number") from None


def _parse_xgb_model(doc: Mapping) -> dict:
    """The flat arrays ``fb_model_create`` takes, from an XGBoost JSON document,
    with the reference loader's checks (src/model/tree.rs:765-890 for the
    learner, :1258-1362 for each tree's arrays and category segments)."""
    learner = doc["learner"]
    booster = learner["gradient_booster"]
    if booster.get("name", "gbtree") != "gbtree":
        raise ValueError(f"only gbtree is supported, this model is {booster.get('name')}")
    objective = learner["objective"]
    obj = objective["name"]
    if obj == "reg:linear":  # objective.rs:144
        obj = "reg:squarederror"
    if obj not in _OBJECTIVES:
        raise ValueError(f"objective {obj!r} is not supported on this engine; supported objectives: "
                         f"{', '.join(_OBJECTIVES)}")
    multi = obj.startswith("multi:")
    lp = learner["learner_model_param"]
    num_class = max(_int_param("num_class", lp.get("num_class", "0") or "0"), 1)
    nt_raw = str(lp.get("num_target", "")).strip()
    num_target = max(_int_param("num_target", nt_raw), 1) if nt_raw else 1
    if num_target > 1:
        raise ValueError(f"multi-target models are not supported (num_target = {num_target})")
    K = max(num_class, num_target)
    gbm = booster["model"]
    trees = gbm["trees"]
    for i, g in enumerate(gbm.get("tree_info", [])):
        if int(g) != i % K:
            raise ValueError(f"tree {i} has tree_info = {g}, not {i} % num_class ({K}); this output group "
                             "layout is not supported")
    for t in trees:
        leaf_vec = str(t.get("tree_param", {}).get("size_leaf_vector", "")).strip()
        if leaf_vec and _int_param("size_leaf_vector", leaf_vec) > 1:
            raise ValueError(f"tree {t.get('id')} has vector leaves (size_leaf_vector = {leaf_vec}); only scalar "
                             "leaves are supported")
    npt = gbm.get("gbtree_model_param", {}).get("num_parallel_tree", "1")
    if _int_param("num_parallel_tree", npt) != 1:
        raise ValueError(f"num_parallel_tree = {npt} (random forest mode) is not supported")
    outputs = _int_param("num_class", objective.get("softmax_multiclass_param", {}).get("num_class", K)) \
        if multi else 1
    if K != outputs or (multi and K < 2):
        raise ValueError(f"num_class = {K} is inconsistent with objective {obj}")
    F = _int_param("num_feature", lp["num_feature"])
    margins = _base_scores(lp["base_score"], multi)
    if multi:
        margins = margins * K if len(margins) == 1 else margins  # an old scalar: K copies
        if len(margins) != K:
            raise ValueError(f"base_score has {len(margins)} values, but num_class = {K}")
    spw = float(objective.get("reg_loss_param", {}).get("scale_pos_weight", "1"))
    ftypes = learner.get("feature_types") or []
    if "c" in ftypes and len(ftypes) != F:
        raise ValueError(f"feature_types has {len(ftypes)} entries, but the model has {F} features")
    cols = {k: [] for k in ("left", "right", "feat", "cond", "dl", "leaf", "gain", "hess", "cat", "coff", "clen")}
    words: list = []
    off = [0]
    for ti, t in enumerate(trees):
        tid = t.get("id", ti)
        n = len(t["left_children"])
        if n == 0:
            raise ValueError(f"tree {tid} has no root node")
        for name in ("right_children", "split_conditions", "split_indices", "default_left"):
            if len(t[name]) != n:
                raise ValueError(f"tree {tid}: {name} length {len(t[name])} does not match node count {n}")
        split_type = [int(v) for v in t.get("split_type") or []]
        if split_type and len(split_type) != n:
            raise ValueError(f"tree {tid}: split_type length {len(split_type)} does not match node count {n}")
        if any(v not in (0, 1) for v in split_type):
            raise ValueError(f"tree {tid}: unknown split_type (0 = numerical, 1 = categorical)")
        split_type = split_type or [0] * n
        nodes, segs, sizes = (t.get(k, []) for k in ("categories_nodes", "categories_segments", "categories_sizes"))
        if not len(nodes) == len(segs) == len(sizes):
            raise ValueError(f"tree {tid}: categories_nodes / segments / sizes have different lengths")
        categories = t.get("categories", [])
        cats_of: dict = {}
        for node, seg, size in zip(nodes, segs, sizes):
            node, seg, size = int(node), int(seg), int(size)
            if seg < 0 or size < 0 or seg + size > len(categories):
                raise ValueError(f"tree {tid}: category segment [{seg}, +{size}) is out of bounds, categories has "
                                 f"{len(categories)} entries")
            if not 0 <= node < n or split_type[node] != 1:
                raise ValueError(f"tree {tid}: categories_nodes contains {node}, which is not a categorical split "
                                 "node")
            cs = [int(c) for c in categories[seg:seg + size]]
            if any(c < 0 for c in cs):
                raise ValueError(f"tree {tid}: node {node} contains a negative category value")
            if any(c >= 1 << 24 for c in cs):
                raise ValueError(f"tree {tid}: node {node} contains a category value above 2^24")
            if node in cats_of:
                raise ValueError(f"tree {tid}: node {node} appears more than once in categories_nodes")
            cats_of[node] = cs
        gains, hesses = t.get("loss_changes", []), t.get("sum_hessian", [])
        for i in range(n):
            left = int(t["left_children"][i])
            is_cat = split_type[i] == 1
            if is_cat and i not in cats_of:
                raise ValueError(f"tree {tid}: node {i} is a categorical split but has no category segment")
            cols["left"].append(left)
            cols["right"].append(int(t["right_children"][i]))
            cols["feat"].append(int(t["split_indices"][i]))
            cols["cond"].append(float(t["split_conditions"][i]))
            cols["dl"].append(int(bool(t["default_left"][i])))
            cols["leaf"].append(float(t["split_conditions"][i]) if left < 0 else 0.0)  # leaves live in split_conditions
            cols["gain"].append(float(gains[i]) if i < len(gains) else 0.0)
            cols["hess"].append(float(hesses[i]) if i < len(hesses) else 0.0)
            cols["cat"].append(int(is_cat))
            cols["coff"].append(len(words))
            w = []
            if is_cat:
                cs = cats_of[i]
                w = [0] * ((max(cs) >> 5) + 1 if cs else 0)
                for c in cs:
                    w[c >> 5] |= 1 << (c & 31)
            words.extend(w)
            cols["clen"].append(len(w))
        off.append(off[-1] + n)
    dt = {"left": np.int32, "right": np.int32, "feat": np.uint32, "cond": np.float32, "dl": np.uint8,
          "leaf": np.float32, "gain": np.float32, "hess": np.float32, "cat": np.uint8, "coff": np.uint32,
          "clen": np.uint32}
    out = {k: np.array(v, dt[k]) for k, v in cols.items()}
    out.update(F=F, objective=obj, K=K if multi else 0, margins=margins, spw=spw, off=np.array(off, np.uint32),
               words=np.array(words if words else [0], np.uint32), n_words=len(words),
               class_margins=np.array(margins, np.float32) if multi else None,
               ftypes=np.array([v == "c" for v in ftypes], np.uint8) if "c" in ftypes else None)
    return out


def _err() -> str:
    return (lib().fb_last_error() or b"").decode()


def _normalize_params(params: Mapping[str, Any], num_boost_round: int) -> dict[str, Any]:
    """Reference python/ferrisboost/__init__.py:180-323 rules for this engine's parameters."""
    out = dict(_DEFAULTS)
    for key, value in dict(params).items():
        canon = _ALIASES.get(key, key)
        if canon not in _DEFAULTS:
            known = ", ".join(sorted(_DEFAULTS) + sorted(_ALIASES))
            raise ValueError(f"unknown parameter {key!r}; supported parameters: {known}")
        out[canon] = value
    if out["objective"] == "reg:linear":  # objective.rs:144: XGBoost's old name of squared error
        out["objective"] = "reg:squarederror"
    if out["objective"] not in _OBJECTIVES:
        raise ValueError(f"objective {out['objective']!r} is not supported on this engine; supported objectives: "
                         f"{', '.join(_OBJECTIVES)}")
    if not 0 < int(out["max_bin"]) <= 65535:
        raise ValueError(f"max_bin must be in 1..=65535, got {out['max_bin']}")
    if num_boost_round < 1:
        raise ValueError(f"num_boost_round must be >= 1, got {num_boost_round}")
    for key in ("max_depth", "max_leaves", "max_bin", "nthread", "seed", "max_cat_to_onehot", "max_cat_threshold",
                "num_class"):
        out[key] = int(out[key])
    out["missing"] = _validate_missing(out["missing"])
    if out["objective"].startswith("multi:") and out["num_class"] < 2:  # objective.rs:331-337
        raise ValueError(f"{out['objective']} requires num_class >= 2, got {out['num_class']}")
    if out["max_leaves"] < 0:
        raise ValueError(f"max_leaves must be >= 0, got {out['max_leaves']}")
    if not 0 <= out["max_depth"] <= 14:
        raise ValueError(f"max_depth must be in 0..=14, got {out['max_depth']}; 0 means a root-only tree")
    if out["grow_policy"] not in ("depthwise", "lossguide"):
        raise ValueError(f"grow_policy must be depthwise or lossguide, got {out['grow_policy']!r}")
    if out["sampling_method"] != "uniform":
        raise ValueError("sampling_method must be uniform on this engine")
    for key in ("colsample_bylevel", "colsample_bynode"):
        if float(out[key]) != 1.0:
            raise ValueError(f"{key} < 1 is not supported on this engine")
    gm = out["gpu_math"] or "exact"
    if gm not in ("exact", "fast"):
        raise ValueError(f'gpu_math must be "exact" or "fast", got {gm!r}')
    out["gpu_math"] = gm
    dev = out["device"]
    if dev is None or dev in ("cuda", "gpu"):
        out["device_index"] = 0
    elif isinstance(dev, str) and dev.startswith("cuda:"):
        out["device_index"] = int(dev.split(":", 1)[1])
    elif dev == "cpu":
        raise ValueError('device="cpu": this engine runs on CUDA devices only; use "cuda" or "cuda:N"')
    else:
        raise ValueError(f'device must be "cuda" or "cuda:N", got {dev!r}')
    for key in ("eta", "lambda", "gamma", "min_child_weight", "alpha", "scale_pos_weight", "subsample",
                "colsample_bytree"):
        out[key] = float(out[key])
        if not math.isfinite(out[key]) or out[key] < 0:
            raise ValueError(f"{key} must be finite and non-negative")
    if not 0.0 < out["subsample"] <= 1.0:
        raise ValueError(f"subsample must be in (0, 1], got {out['subsample']}")
    if not 0.0 < out["colsample_bytree"] <= 1.0:
        raise ValueError(f"colsample_bytree must be in (0, 1], got {out['colsample_bytree']}")
    out["max_delta_step"] = 0.0 if out["max_delta_step"] is None else float(out["max_delta_step"])
    if not math.isfinite(out["max_delta_step"]) or out["max_delta_step"] < 0:
        raise ValueError(f"max_delta_step must be finite and non-negative, got {out['max_delta_step']}")
    if out["base_score"] is not None:
        out["base_score"] = float(out["base_score"])
    for key in ("max_cat_to_onehot", "max_cat_threshold"):
        if out[key] < 1:
            raise ValueError(f"{key} must be >= 1, got {out[key]}")
    out["monotone_constraints"] = _normalize_monotone(out["monotone_constraints"])
    out["num_boost_round"] = int(num_boost_round)
    return out


def _monotone_sign(value: Any, where: str) -> int:
    """python/ferrisboost/__init__.py:386-390: an integer (not a bool), of
    which only the sign counts (XGBoost reads 2 as 1 and -3 as -1)."""
    if isinstance(value, bool) or not isinstance(value, (int, np.integer)):
        raise ValueError(f"monotone_constraints {where} must be an integer (1 / 0 / -1), got {value!r}")
    return int(np.sign(int(value)))


def _normalize_monotone(mc: Any) -> "list[int] | dict[str, int] | None":
    """python/ferrisboost/__init__.py:393-419: a tuple / list / array by
    position, a "(1,0,-1)" string, or {column name: direction}; shorter than
    the feature count means 0 for the rest, and all zeros is no constraint."""
    if mc is None:
        return None
    if isinstance(mc, str):
        text = mc.strip()
        if not (text.startswith("(") and text.endswith(")")):
            raise ValueError(f'a monotone_constraints string must look like "(1,0,-1)", got {mc!r}')
        body = text[1:-1].strip()
        try:
            values = [int(v) for v in body.split(",")] if body else []
        except ValueError:
            raise ValueError(f"monotone_constraints string contains a non-integer: {mc!r}") from None
        return [_monotone_sign(v, "element") for v in values]
    if isinstance(mc, Mapping):
        for name in mc:
            if not isinstance(name, str):
                raise ValueError(f"monotone_constraints dict keys must be column name strings, got {name!r}")
        return {name: _monotone_sign(v, f"value for column {name!r}") for name, v in mc.items()}
    if isinstance(mc, (list, tuple, np.ndarray)):
        return [_monotone_sign(v, "element") for v in np.asarray(mc, dtype=object).ravel()]
    raise ValueError('monotone_constraints must be a tuple/list, a "(1,0,-1)" string or a {column name: direction} '
                     f"dict, got {type(mc).__name__}")


def _positional_monotone(mc: "list[int] | dict[str, int] | None", names, n_features: int):
    """Constraints by feature position (python/ferrisboost/__init__.py:
    422-426 and :1344-1350 for names; training/mod.rs:1508-1512 for the
    length)."""
    if isinstance(mc, dict):
        if not names:
            raise ValueError("monotone_constraints given by column name needs column names: a numpy array has none; "
                             "use a positional tuple, or a pyarrow Table / a file with a header")
        unknown = [k for k in mc if k not in names]
        if unknown:
            raise ValueError(f"monotone_constraints columns {unknown} are not feature columns; feature columns: "
                             f"{list(names)}")
        mc = [mc.get(n, 0) for n in names]
    if mc is None:
        return None
    if len(mc) > n_features:
        raise ValueError(f"monotone_constraints has {len(mc)} entries, but there are only {n_features} features")
    mono = np.zeros(n_features, dtype=np.int8)
    mono[:len(mc)] = mc
    return mono


def _fb_params(p: Mapping[str, Any]) -> _lib.FbParams:
    fp = _lib.FbParams()
    lib().fb_default_params(C.byref(fp))
    fp.objective = _OBJECTIVES[p["objective"]]
    fp.grow_policy = 1 if p["grow_policy"] == "lossguide" else 0
    fp.max_depth = p["max_depth"]
    fp.max_leaves = p["max_leaves"]
    fp.max_bin = p["max_bin"]
    fp.eta = p["eta"]
    fp.reg_lambda = p["lambda"]
    fp.gamma = p["gamma"]
    fp.min_child_weight = p["min_child_weight"]
    fp.alpha = p["alpha"]
    fp.max_delta_step = p["max_delta_step"]
    fp.scale_pos_weight = p["scale_pos_weight"]
    fp.subsample = p["subsample"]
    fp.colsample_bytree = p["colsample_bytree"]
    fp.base_score = float("nan") if p["base_score"] is None else p["base_score"]
    fp.seed = p["seed"]
    fp.max_cat_to_onehot = p["max_cat_to_onehot"]
    fp.max_cat_threshold = p["max_cat_threshold"]
    fp.nthread = p["nthread"]
    fp.gpu_math = 1 if p["gpu_math"] == "fast" else 0
    fp.device = p["device_index"]
    fp.num_class = p["num_class"] if p["objective"].startswith("multi:") else 0
    return fp


def _validate_missing(missing: Any) -> float:
    """src/source/mod.rs:218-235 validate_missing: NaN (no sentinel) or a
    finite float32 other than f32::MAX.  +-inf and f32::MAX never occur in
    features (they are rejected there), so a sentinel equal to one of them, or
    one that overflows float32, is refused."""
    m = float(missing)
    if math.isnan(m):
        return m
    with np.errstate(over="ignore"):
        narrowed = np.float32(m)
    if not np.isfinite(narrowed) or narrowed == np.finfo(np.float32).max:
        raise ValueError(f"missing={missing} is not allowed: it must be NaN or a finite float32 value (+/-inf and "
                         "f32::MAX are reserved and rejected in features, so they cannot be the missing marker; "
                         "pick a different sentinel)")
    return float(narrowed)


def _as_matrix(x: Any, missing: float = float("nan")) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    if a.ndim != 2:
        raise ValueError(f"data must be a 2-D array, got shape {a.shape}")
    missing = _validate_missing(missing)
    if not math.isnan(missing):
        a = np.where(a == np.float32(missing), np.float32("nan"), a).astype(np.float32)
    return a


def _feature_flags(feature_types: Sequence[str] | None, n: int) -> np.ndarray | None:
    if feature_types is None:
        return None
    ft = list(feature_types)
    if len(ft) != n:
        raise ValueError(f"feature_types has {len(ft)} entries, the data has {n} features")
    bad = [t for t in ft if t not in ("c", "q", "float", "int", "i")]
    if bad:
        raise ValueError(f"feature_types entries must be 'c' or 'q', got {bad[0]!r}")
    flags = np.array([t == "c" for t in ft], dtype=np.uint8)
    return flags if flags.any() else None


class Shard(NamedTuple):
    """One rank's part of a row-sharded run (see ``ferrisboost_b200.distributed``)."""
    row_offset: int       # global index of this rank's first row
    n_rows_global: int    # rows over all ranks
    nccl_id: bytes        # fbgpu_nccl_unique_id of rank 0, 128 bytes (unused with comm)
    nranks: int
    rank: int
    base_score: float     # over all rows (fb_initial_base_score) or the given base_score
    timeout_ms: int = 120000
    comm: Any = None      # a distributed.Communicator started ahead (its initialization overlaps data preparation)
    class_margins: Any = None  # multiclass: the K base margins over all rows (fb_class_margins)


class Dataset:
    """Quantized training data: cuts from the weighted quantile sketch and
    column blocks of u8/u16 bins (the reference's DenseSource)."""

    def __init__(self, data: Any, max_bin: int = 255, weight: Any = None, feature_types=None, nthread: int = 0,
                 missing: float = float("nan"), cuts: tuple[np.ndarray, np.ndarray] | None = None,
                 device: int | None = None):
        """``cuts`` = (cut values, F+1 offsets) bins the rows with given cuts
        (validation data, or one row shard of a multi-GPU run) instead of
        sketching them.  ``device`` = N sketches and quantizes on CUDA device
        N and keeps the bins there (the same cuts and bins as the host
        preparation; a booster on that device trains from them in place).
        ``data`` may also be a ``columnar.Columns`` (decoded Parquet / Arrow
        feature columns, column-major), which the device path ingests as is."""
        cols = data if isinstance(data, columnar.Columns) else None
        if cols is not None:
            X = cols.X
            self.n_features, self.n_rows = X.shape
            self.feature_names = list(cols.names)
            if feature_types is None and cols.categorical is not None:
                feature_types = ["c" if c else "q" for c in cols.categorical]
        else:
            X = _as_matrix(data, missing)
            self.n_rows, self.n_features = X.shape
            self.feature_names = None
        w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
        cat = _feature_flags(feature_types, self.n_features)
        self.categorical = cat
        self.device = device
        if device is not None:
            cv = off = None
            if cuts is not None:
                cv, off = self._check_cuts(cuts)
                cv = cv if cv.size else np.zeros(1, np.float32)
            make = lib().fb_dataset_on_device_columns if cols is not None else lib().fb_dataset_on_device
            self._h = make(_lib.ptr(X, C.c_float), self.n_rows, self.n_features, max_bin, _lib.ptr(w, C.c_float),
                           _lib.ptr(cat, C.c_uint8), _lib.ptr(cv, C.c_float), _lib.ptr(off, C.c_uint32), nthread,
                           int(device))
            if not self._h:
                raise ValueError(_err())
            return
        if cols is not None:  # host preparation reads rows
            X = np.ascontiguousarray(X.T)
        if cuts is None:
            self._h = lib().fb_dataset_from_dense(_lib.ptr(X, C.c_float), X.shape[0], X.shape[1], max_bin,
                                                  _lib.ptr(w, C.c_float), _lib.ptr(cat, C.c_uint8), nthread)
        else:
            cv, off = self._check_cuts(cuts)
            self._h = lib().fb_dataset_with_cuts(_lib.ptr(X, C.c_float), X.shape[0], X.shape[1],
                                                 _lib.ptr(cv if cv.size else np.zeros(1, np.float32), C.c_float),
                                                 _lib.ptr(off, C.c_uint32), _lib.ptr(cat, C.c_uint8), nthread)
        if not self._h:
            raise ValueError(_err())

    def _check_cuts(self, cuts):
        cv = np.ascontiguousarray(cuts[0], dtype=np.float32)
        off = np.ascontiguousarray(cuts[1], dtype=np.uint32)
        if off.shape != (self.n_features + 1,) or int(off[-1]) != cv.size or np.any(np.diff(off.astype(np.int64)) < 0):
            raise ValueError("cuts must be (values, offsets) with F+1 non-decreasing offsets ending at len(values)")
        return cv, off

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().fb_dataset_free(h)
            except TypeError:  # interpreter shutdown: module globals already cleared
                pass
            self._h = None

    def cuts(self):
        n = lib().fb_dataset_cuts(self._h, None, None, 0)
        cuts = np.zeros(max(n, 1), dtype=np.float32)
        off = np.zeros(self.n_features + 1, dtype=np.uint32)
        lib().fb_dataset_cuts(self._h, _lib.ptr(cuts, C.c_float), _lib.ptr(off, C.c_uint32), n)
        return cuts[:n], off

    def column(self, f: int) -> np.ndarray:
        out = np.zeros(self.n_rows, dtype=np.uint16)
        if lib().fb_dataset_column(self._h, f, _lib.ptr(out, C.c_uint16)):
            raise IndexError(f)
        return out


class Booster:
    """A training run on one CUDA device; ``update(k)`` adds k trees."""

    def __init__(self, params: Mapping[str, Any], dataset: Dataset, label: Any, weight: Any = None,
                 shard: "Shard | None" = None):
        """``shard`` makes this booster one rank of a row-sharded multi-GPU run
        (``ferrisboost_b200.distributed``); ``dataset``, ``label`` and
        ``weight`` then hold that rank's rows only."""
        p = _normalize_params(params, 1)
        y = np.ascontiguousarray(label, dtype=np.float32)
        if y.shape != (dataset.n_rows,):
            raise ValueError(f"label has shape {y.shape}, expected ({dataset.n_rows},)")
        w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
        self.params = p
        fp = _fb_params(p)
        mono = _positional_monotone(p["monotone_constraints"], getattr(dataset, "feature_names", None),
                                    dataset.n_features)
        if mono is not None:
            fp.monotone = _lib.ptr(mono, C.c_int8)
        self._keep = (y, w, mono, dataset)
        if shard is None:
            self._h = lib().fb_booster_create(dataset._h, _lib.ptr(y, C.c_float), _lib.ptr(w, C.c_float),
                                              C.byref(fp))
        elif shard.comm is not None:
            fp.base_score = shard.base_score
            if shard.class_margins is not None:
                cm = np.ascontiguousarray(shard.class_margins, dtype=np.float32)
                self._keep = self._keep + (cm,)
                fp.class_margins = _lib.ptr(cm, C.c_float)
            self._keep = self._keep + (shard.comm,)
            self._h = lib().fb_booster_create_sharded_comm(
                dataset._h, _lib.ptr(y, C.c_float), _lib.ptr(w, C.c_float), C.byref(fp), shard.row_offset,
                shard.n_rows_global, shard.comm.handle, shard.nranks, shard.rank)
        else:
            fp.base_score = shard.base_score
            if shard.class_margins is not None:
                cm = np.ascontiguousarray(shard.class_margins, dtype=np.float32)
                self._keep = self._keep + (cm,)
                fp.class_margins = _lib.ptr(cm, C.c_float)
            nid = np.frombuffer(shard.nccl_id, dtype=np.uint8).copy()
            self._h = lib().fb_booster_create_sharded(
                dataset._h, _lib.ptr(y, C.c_float), _lib.ptr(w, C.c_float), C.byref(fp), shard.row_offset,
                shard.n_rows_global, _lib.ptr(nid, C.c_uint8), shard.nranks, shard.rank, shard.timeout_ms)
        if not self._h:
            raise ValueError(_err())

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().fb_booster_free(h)
            except TypeError:  # interpreter shutdown: module globals already cleared
                pass
            self._h = None

    def update(self, n_rounds: int = 1) -> None:
        if lib().fb_booster_update(self._h, n_rounds):
            raise RuntimeError(_err())

    def set_stats(self, on: bool = True) -> None:
        lib().fb_booster_set_stats(self._h, int(on))

    def timing(self) -> dict:
        t = np.zeros(8, dtype=np.float64)
        lib().fb_booster_timing(self._h, _lib.ptr(t, C.c_double))
        keys = ("wall_ms", "gradient_ms", "tree_ms", "device_ms", "hist_ms", "hist_launches", "hist_bytes", "trees")
        out = {k: float(v) for k, v in zip(keys, t)}
        # of hist_ms: the per-level histogram all-reduces of a row-sharded run
        out["comm_ms"] = float(lib().fb_booster_collective_ms(self._h))
        out["hist_updates"] = float(lib().fb_booster_hist_updates(self._h))
        return out

    def margins(self) -> np.ndarray:
        """Training margins: n values, or K x n (class-major) for multiclass."""
        n = self._keep[3].n_rows
        K = self.params["num_class"] if self.params["objective"].startswith("multi:") else 1
        out = np.zeros(n if K == 1 else (K, n), dtype=np.float32)
        if lib().fb_booster_margins(self._h, _lib.ptr(out, C.c_float)):
            raise RuntimeError(_err())
        return out

    def model(self) -> "Model":
        m = Model(lib().fb_booster_model(self._h), self.params)
        return m


class Model:
    """A trained model (the reference's ``Model``)."""

    def __init__(self, handle, params: Mapping[str, Any] | None = None):
        if not handle:
            raise RuntimeError(_err())
        self._h = handle
        self.params = dict(params or {})
        # column names of a Parquet / Arrow training set (src/model/tree.rs:244):
        # written to the JSON and used to bind prediction columns by name
        self.feature_names: list[str] | None = None

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().fb_model_free(h)
            except TypeError:  # interpreter shutdown: module globals already cleared
                pass
            self._h = None

    @property
    def num_trees(self) -> int:
        return lib().fb_model_num_trees(self._h)

    @property
    def n_features(self) -> int:
        return lib().fb_model_num_features(self._h)

    @property
    def num_outputs(self) -> int:
        """num_class for multi:softprob / multi:softmax models, else 1."""
        return lib().fb_model_num_outputs(self._h)

    def _device(self, device=None) -> int:
        d = device if device is not None else self.params.get("device")
        if d is None or d in ("cuda", "gpu"):
            return int(self.params.get("device_index", 0))
        if isinstance(d, int):
            return d
        return int(str(d).split(":", 1)[1])

    def device_handle(self, device=None):
        """The model's device copy (an include/fbgpu.h ``fbgpu_model*``) for
        fbgpu_predict_device / fbgpu_shap_device on rows already in HBM."""
        h = lib().fb_model_device(self._h, self._device(device))
        if not h:
            raise RuntimeError(_err())
        return h

    def to_json(self) -> bytes:
        n = lib().fb_model_json(self._h, None, 0)
        buf = C.create_string_buffer(n)
        lib().fb_model_json(self._h, buf, n)
        out = buf.raw[:n]
        if self.feature_names:
            names = json.dumps(list(self.feature_names), ensure_ascii=False, separators=(",", ":"))
            out = out.replace(b'"feature_names":[]', b'"feature_names":' + names.encode("utf-8"), 1)
        return out

    @staticmethod
    def load_model(source: "str | os.PathLike | bytes", device=None) -> "Model":
        """A model from XGBoost-compatible JSON: a path or the JSON bytes (the
        reference's ``Model.load_model``, src/model/tree.rs:754-1460).  Models
        of this engine and XGBoost models of its objectives (reg:squarederror,
        binary:logistic, multi:softprob, multi:softmax) load; ``save_model`` of
        the result writes the same JSON back.  What the reference rejects is
        rejected here with ValueError: another booster, forests, multi-target
        models and vector leaves, a num_class that disagrees with the
        objective, trees out of the t % num_class order, malformed arrays or
        category segments, and anything that is not a tree (checked by
        ``fb_model_create``)."""
        if isinstance(source, (bytes, bytearray)):
            doc = json.loads(source)
        else:
            with open(os.fspath(source), "rb") as f:
                doc = json.load(f)
        a = _parse_xgb_model(doc)
        h = lib().fb_model_create(a["F"], _OBJECTIVES[a["objective"]], float(a["margins"][0]), a["spw"], a["K"],
                                  _lib.ptr(a["class_margins"], C.c_float), _lib.ptr(a["ftypes"], C.c_uint8),
                                  len(a["off"]) - 1, _lib.ptr(a["off"], C.c_uint32), _lib.ptr(a["left"], C.c_int32),
                                  _lib.ptr(a["right"], C.c_int32), _lib.ptr(a["feat"], C.c_uint32),
                                  _lib.ptr(a["cond"], C.c_float), _lib.ptr(a["dl"], C.c_uint8),
                                  _lib.ptr(a["leaf"], C.c_float), _lib.ptr(a["gain"], C.c_float),
                                  _lib.ptr(a["hess"], C.c_float), _lib.ptr(a["cat"], C.c_uint8),
                                  _lib.ptr(a["coff"], C.c_uint32), _lib.ptr(a["clen"], C.c_uint32),
                                  _lib.ptr(a["words"], C.c_uint32), a["n_words"])
        if not h:
            raise ValueError(_err())
        params = {"objective": a["objective"], "num_class": a["K"], "missing": float("nan")}
        if device is not None:
            params["device"] = device
        m = Model(h, params)
        m.feature_names = list(doc["learner"].get("feature_names") or []) or None
        return m

    def save_model(self, path: str | os.PathLike) -> None:
        """XGBoost-compatible JSON (reference src/model/model_io.rs: atomic write)."""
        path = os.fspath(path)
        tmp = path + ".tmp"
        with open(tmp, "wb") as f:
            f.write(self.to_json())
        os.replace(tmp, path)

    def tree(self, t: int) -> dict:
        n = lib().fb_model_tree(self._h, t, *([None] * 10))
        if n < 0:
            raise IndexError(t)
        a = {"left": np.zeros(n, np.int32), "right": np.zeros(n, np.int32), "feat": np.zeros(n, np.uint32),
             "cond": np.zeros(n, np.float32), "default_left": np.zeros(n, np.uint8), "leaf": np.zeros(n, np.float32),
             "is_leaf": np.zeros(n, np.uint8), "gain": np.zeros(n, np.float32), "hess": np.zeros(n, np.float32),
             "cats": np.zeros((n, 8), np.uint32)}
        ct = [C.c_int32, C.c_int32, C.c_uint32, C.c_float, C.c_uint8, C.c_float, C.c_uint8, C.c_float, C.c_float,
              C.c_uint32]
        lib().fb_model_tree(self._h, t, *[_lib.ptr(v, c) for v, c in zip(a.values(), ct)])
        return a

    def _rows(self, data: Any) -> np.ndarray:
        """Row-major f32 rows for the prediction entry points."""
        missing = _validate_missing(self.params.get("missing", float("nan")))
        specs = columnar.path_specs(data)
        table = None if specs is not None else columnar.arrow_table(data)
        if specs is None and table is None:
            return _as_matrix(data, missing)
        if not self.feature_names:
            raise ValueError("this model has no feature names to bind Parquet / Arrow columns to; pass an array")
        if specs is not None:
            X = columnar.read_file_features(specs, self.feature_names, missing)
        else:
            X = columnar.read_table(table, False, None, missing, order=list(self.feature_names), scoring=True).X
        return np.ascontiguousarray(X.T)

    def predict(self, data: Any, output_margin: bool = False, pred_contribs: bool = False, device=None, *,
                approx_contribs: bool = False, pred_interactions: bool = False, pred_leaf: bool = False):
        """Predictions (probabilities for binary:logistic unless output_margin),
        or (the reference's _core.Model.predict options): SHAP contributions
        n x (F+1) with the bias last (pred_contribs; Saabas values with
        approx_contribs), SHAP interaction values n x (F+1) x (F+1)
        (pred_interactions), or the leaf node index of every tree, n x n_trees
        as float32 (pred_leaf).  Parquet paths and pyarrow tables bind their
        columns to the model's feature names (any column order; other columns
        of a file, such as the label, are not read)."""
        X = self._rows(data)
        if X.shape[1] != self.n_features:
            raise ValueError(f"data has {X.shape[1]} features, the model has {self.n_features}")
        if sum(bool(v) for v in (pred_contribs, pred_interactions, pred_leaf)) > 1:
            raise ValueError("pred_contribs, pred_interactions and pred_leaf are mutually exclusive")
        dev = self._device(device)
        K = self.num_outputs
        groups = (K,) if K > 1 else ()  # multiclass: a class axis after the row (explain.rs:704-727)
        kind = None
        nc = X.shape[1] + 1
        if pred_leaf:
            kind, shape = 0, (X.shape[0], self.num_trees)
        elif pred_contribs and approx_contribs:
            kind, shape = 1, (X.shape[0], *groups, nc)
        elif pred_interactions:
            kind, shape = 2, (X.shape[0], *groups, nc, nc)
        if kind is not None:
            out = np.zeros(shape, dtype=np.float32)
            if lib().fb_model_explain(self._h, kind, _lib.ptr(X, C.c_float), X.shape[0], _lib.ptr(out, C.c_float),
                                      dev):
                raise RuntimeError(_err())
            return out
        if pred_contribs:
            out = np.zeros((X.shape[0], *groups, nc), dtype=np.float32)
            if lib().fb_model_shap(self._h, _lib.ptr(X, C.c_float), X.shape[0], _lib.ptr(out, C.c_float), dev):
                raise RuntimeError(_err())
            return out
        out = np.zeros((X.shape[0], *groups), dtype=np.float32)
        if lib().fb_model_predict(self._h, _lib.ptr(X, C.c_float), X.shape[0], _lib.ptr(out, C.c_float), dev):
            raise RuntimeError(_err())
        objective = self.params.get("objective", "binary:logistic")
        if output_margin or objective == "reg:squarederror":
            return out
        if K > 1:  # objective.rs:1260-1333: softprob -> probabilities, softmax -> class index
            classes = np.zeros(X.shape[0], dtype=np.float32)
            if lib().fb_model_transform(self._h, _lib.ptr(out, C.c_float), X.shape[0], _lib.ptr(classes, C.c_float)):
                raise RuntimeError(_err())
            return classes if objective == "multi:softmax" else out
        return (1.0 / (1.0 + np.exp(-out.astype(np.float64)))).astype(np.float32)


def train(params: Mapping[str, Any], data: Any, label: Any = None, num_boost_round: int = 10, weight: Any = None,
          feature_types: Sequence[str] | None = None, quiet: bool = True, header: bool = True) -> Model:
    """Train a model (reference python/ferrisboost/__init__.py:1090 ``train``).

    ``data`` is a 2-D array with ``label`` (and ``weight``) arrays; a
    ``.parquet`` / ``.csv`` path, a list of paths, a directory or a glob
    pattern with ``label`` (and ``weight``) naming columns of the files (a
    headerless CSV, ``header=False``: column indices); or a pyarrow
    Table / RecordBatch / RecordBatchReader with ``label`` an array
    (``columnar`` has the decode rules).  Columnar inputs record their column
    names as the model's feature names."""
    p = _normalize_params(params, num_boost_round)
    specs = columnar.path_specs(data)
    table = None if specs is not None else columnar.arrow_table(data)
    if specs is not None:
        col = str if header else int
        kind = "the name" if header else "the index"
        if not isinstance(label, col) or isinstance(label, bool):
            raise ValueError(f"for file input, label must be {kind} of a column of the file")
        if weight is not None and (not isinstance(weight, col) or isinstance(weight, bool)):
            raise ValueError(f"for file input, weight must be {kind} of a column of the file")
        data = columnar.read_files(specs, label, weight, feature_types, p["missing"], header=header)
        label, weight, feature_types = data.label, data.weight, None
    elif table is not None:
        data = columnar.read_table(table, p["enable_categorical"], feature_types, p["missing"])
        feature_types = None
    if label is None:
        raise ValueError("label is required for array input")
    from ._trace import PhaseTrace
    trace = PhaseTrace("train")
    ds = Dataset(data, max_bin=p["max_bin"], weight=weight, feature_types=feature_types, nthread=p["nthread"],
                 missing=p["missing"], device=p["device_index"])
    trace("dataset (upload, sketch, bins)")
    b = Booster(params, ds, label, weight)
    trace("booster")
    b.update(num_boost_round)
    trace("rounds")
    m = b.model()
    m.params = p
    m.feature_names = ds.feature_names or None
    trace("model")
    del b, ds
    trace("release")
    return m
