"""ctypes binding of oracle/_build/librefcpu.so (test infrastructure only)."""
import ctypes as C
import json
import math
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "librefcpu.so"


def build() -> None:
    """Compile the oracle with its Makefile (g++, OpenMP, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


class rc_params(C.Structure):
    _fields_ = [
        ("objective", C.c_int32), ("grow_policy", C.c_int32), ("n_rounds", C.c_uint32),
        ("max_depth", C.c_uint32), ("max_leaves", C.c_uint32), ("max_bin", C.c_uint32),
        ("eta", C.c_float), ("reg_lambda", C.c_float), ("gamma", C.c_float),
        ("min_child_weight", C.c_float), ("alpha", C.c_float), ("max_delta_step", C.c_float),
        ("scale_pos_weight", C.c_float), ("subsample", C.c_float), ("colsample_bytree", C.c_float),
        ("base_score", C.c_float), ("seed", C.c_uint64), ("max_cat_to_onehot", C.c_uint32),
        ("max_cat_threshold", C.c_uint32), ("nthread", C.c_int32),
        ("monotone", C.POINTER(C.c_int8)), ("categorical", C.POINTER(C.c_uint8)), ("num_class", C.c_uint32),
    ]


class rc_split(C.Structure):
    _fields_ = [
        ("found", C.c_uint32), ("feat", C.c_uint32), ("bin", C.c_uint32), ("missing_left", C.c_uint32),
        ("gain", C.c_float), ("pad", C.c_float), ("left_g", C.c_int64), ("left_h", C.c_int64),
        ("right_g", C.c_int64), ("right_h", C.c_int64), ("cats", C.c_uint32 * 8),
    ]


_P = C.c_void_p
OBJECTIVES = {"reg:squarederror": 0, "binary:logistic": 1, "multi:softprob": 2, "multi:softmax": 3}


def _ptr(a, ctype):
    return a.ctypes.data_as(C.POINTER(ctype)) if a is not None else None


class RefCPU:
    """The CPU oracle: train / predict / SHAP / JSON and component kernels."""

    def __init__(self, path=LIB_PATH):
        if not pathlib.Path(path).exists():
            build()
        lib = C.CDLL(str(path))
        lib.rc_train.restype = _P
        lib.rc_train.argtypes = [C.POINTER(C.c_float), C.c_uint64, C.c_uint32, C.POINTER(C.c_float),
                                 C.POINTER(C.c_float), C.POINTER(rc_params)]
        lib.rc_last_error.restype = C.c_char_p
        lib.rc_train_sharded.restype = _P
        lib.rc_train_sharded.argtypes = [C.POINTER(C.c_float), C.c_uint64, C.c_uint32, C.POINTER(C.c_float),
                                         C.POINTER(C.c_float), C.POINTER(rc_params), C.c_int32, C.c_int32]
        lib.rc_last_timing.argtypes = [C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_int32]
        lib.rc_last_timing.restype = C.c_int32
        lib.rc_model_free.argtypes = [_P]
        lib.rc_model_num_trees.argtypes = [_P]
        lib.rc_model_num_trees.restype = C.c_uint32
        lib.rc_model_num_outputs.argtypes = [_P]
        lib.rc_model_num_outputs.restype = C.c_uint32
        lib.rc_softmax_gradients.argtypes = [C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_float),
                                             C.c_uint64, C.c_uint32, C.POINTER(C.c_float)]
        lib.rc_class_margins.argtypes = [C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_uint64, C.c_uint32,
                                         C.POINTER(C.c_float)]
        lib.rc_model_json.argtypes = [_P, C.c_char_p, C.c_int64]
        lib.rc_model_json.restype = C.c_int64
        lib.rc_model_base_margin.argtypes = [_P]
        lib.rc_model_base_margin.restype = C.c_float
        lib.rc_predict_margin.argtypes = [_P, C.POINTER(C.c_float), C.c_uint64, C.POINTER(C.c_float), C.c_int32]
        lib.rc_shap.argtypes = [_P, C.POINTER(C.c_float), C.c_uint64, C.POINTER(C.c_float), C.c_int32]
        for name in ("rc_pred_leaf", "rc_pred_approx", "rc_pred_interactions"):
            getattr(lib, name).argtypes = [_P, C.POINTER(C.c_float), C.c_uint64, C.POINTER(C.c_float), C.c_int32]
        lib.rc_sketch.argtypes = [C.POINTER(C.c_float), C.c_uint64, C.c_uint32, C.c_uint32, C.POINTER(C.c_float),
                                  C.POINTER(C.c_uint8), C.POINTER(C.c_float), C.POINTER(C.c_uint32), C.c_uint64,
                                  C.c_int32]
        lib.rc_sketch.restype = C.c_int64
        lib.rc_quantize.argtypes = [C.POINTER(C.c_float), C.c_uint64, C.c_uint32, C.POINTER(C.c_float),
                                    C.POINTER(C.c_uint32), C.POINTER(C.c_uint8), C.POINTER(C.c_uint16)]
        lib.rc_quantizer.argtypes = [C.POINTER(C.c_float), C.c_uint64, C.c_uint64, C.POINTER(C.c_double)]
        lib.rc_quantizer.restype = C.c_int
        lib.rc_pow2_scales.argtypes = [C.POINTER(C.c_float), C.c_uint64, C.c_uint64, C.POINTER(C.c_double)]
        lib.rc_pow2_scales.restype = None
        lib.rc_pow2_scale_digest.argtypes = [C.c_uint32, C.c_uint32, C.c_uint64]
        lib.rc_pow2_scale_digest.restype = C.c_uint64
        lib.rc_to_fixed.argtypes = [C.POINTER(C.c_float), C.c_uint64, C.POINTER(C.c_double),
                                    C.POINTER(C.c_int64), C.POINTER(C.c_int64)]
        lib.rc_hist.argtypes = [C.POINTER(C.c_uint16), C.c_uint64, C.c_uint32, C.POINTER(C.c_uint32),
                                C.POINTER(C.c_uint16), C.POINTER(C.c_int64), C.POINTER(C.c_uint32), C.c_uint64,
                                C.POINTER(C.c_int64)]
        lib.rc_best_split.argtypes = [C.POINTER(C.c_int64), C.c_uint32, C.POINTER(C.c_uint32),
                                      C.POINTER(C.c_int64), C.POINTER(C.c_double), C.POINTER(rc_params),
                                      C.c_float, C.c_float, C.POINTER(C.c_uint8), C.POINTER(rc_split)]
        lib.rc_default_params.argtypes = [C.POINTER(rc_params)]
        lib.rc_sample_features.argtypes = [C.c_uint32, C.c_float, C.c_uint64, C.c_uint64, C.POINTER(C.c_uint32)]
        lib.rc_sample_features.restype = C.c_uint32
        lib.rc_rows_selected.argtypes = [C.c_uint64, C.c_float, C.c_uint64, C.c_uint64, C.POINTER(C.c_uint8)]
        lib.rc_model_load.restype = _P
        lib.rc_model_load.argtypes = [C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                      C.POINTER(C.c_uint32), C.POINTER(C.c_float), C.POINTER(C.c_uint8),
                                      C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.c_uint32, C.c_int32, C.c_float,
                                      C.POINTER(C.c_float), C.c_uint32, C.c_float, C.POINTER(C.c_uint8)]
        self.lib = lib

    # ---------------------------------------------------------------- params
    def params(self, **kw) -> rc_params:
        p = rc_params()
        self.lib.rc_default_params(C.byref(p))
        keep = []
        for k, v in kw.items():
            if k == "objective":
                p.objective = OBJECTIVES[v] if isinstance(v, str) else int(v)
            elif k == "grow_policy":
                p.grow_policy = {"depthwise": 0, "lossguide": 1}[v] if isinstance(v, str) else int(v)
            elif k in ("lambda", "reg_lambda"):
                p.reg_lambda = v
            elif k in ("learning_rate", "eta"):
                p.eta = v
            elif k == "base_score":
                p.base_score = float("nan") if v is None else v
            elif k == "monotone_constraints":
                a = np.ascontiguousarray(v, dtype=np.int8)
                keep.append(a)
                p.monotone = _ptr(a, C.c_int8)
            elif k == "categorical":
                a = np.ascontiguousarray(v, dtype=np.uint8)
                keep.append(a)
                p.categorical = _ptr(a, C.c_uint8)
            elif k in ("num_boost_round", "n_rounds"):
                p.n_rounds = v
            else:
                setattr(p, k, v)
        p._keep = keep
        return p

    # ---------------------------------------------------------------- model
    def train(self, X, y, w=None, **kw):
        X = np.ascontiguousarray(X, dtype=np.float32)
        y = np.ascontiguousarray(y, dtype=np.float32)
        w = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
        p = self.params(**kw)
        h = self.lib.rc_train(_ptr(X, C.c_float), X.shape[0], X.shape[1], _ptr(y, C.c_float),
                              _ptr(w, C.c_float), C.byref(p))
        if not h:
            raise RuntimeError(self.lib.rc_last_error().decode())
        return RefModel(self, h, X.shape[1])

    def train_sharded(self, X, y, w=None, ranks=2, feature_sharded=False, **kw):
        """train() with rows sharded over `ranks` threads as ranks (the device
        engine's multi-GPU algorithm on the CPU); must give train()'s model."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        y = np.ascontiguousarray(y, dtype=np.float32)
        w = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
        p = self.params(**kw)
        h = self.lib.rc_train_sharded(_ptr(X, C.c_float), X.shape[0], X.shape[1], _ptr(y, C.c_float),
                                      _ptr(w, C.c_float), C.byref(p), ranks, int(feature_sharded))
        if not h:
            raise RuntimeError(self.lib.rc_last_error().decode())
        return RefModel(self, h, X.shape[1])

    def load_json(self, doc):
        """A model from XGBoost JSON text (bytes or str): the document's tree
        arrays are parsed here and handed to rc_model_load.  Used to explain or
        predict with a model trained elsewhere (the device engine) on the
        oracle; writing it back with json() reproduces the document."""
        d = json.loads(doc)
        learner = d["learner"]
        trees = learner["gradient_booster"]["model"]["trees"]
        obj_name = learner["objective"]["name"]
        objective = OBJECTIVES.get(obj_name, 0 if obj_name == "reg:linear" else None)
        if objective is None:
            raise ValueError(f"objective {obj_name!r} is not supported by the oracle")
        nf = int(learner["learner_model_param"]["num_feature"])
        num_class = int(learner["learner_model_param"].get("num_class", "0"))
        base = learner["learner_model_param"]["base_score"]
        margins = None
        if base.startswith("["):
            margins = np.array([float(v) for v in base.strip("[]").split(",")], dtype=np.float32)
            base_score = 0.5
        else:
            base_score = float(base)
        spw = float(learner["objective"].get("reg_loss_param", {}).get("scale_pos_weight", "1"))
        ft = learner.get("feature_types") or []
        ftypes = np.array([t == "c" for t in ft], np.uint8) if ft else None
        off = [0]
        cols = {k: [] for k in ("left", "right", "feat", "value", "dl", "gain", "hess")}
        cat_off, cat_len, cats = [], [], []
        for t in trees:
            nn = len(t["left_children"])
            off.append(off[-1] + nn)
            cols["left"] += t["left_children"]
            cols["right"] += t["right_children"]
            cols["feat"] += t["split_indices"]
            cols["value"] += t["split_conditions"]
            cols["dl"] += t["default_left"]
            cols["gain"] += t["loss_changes"]
            cols["hess"] += t["sum_hessian"]
            per_node = {}
            for node, seg, size in zip(t["categories_nodes"], t["categories_segments"], t["categories_sizes"]):
                per_node[node] = t["categories"][seg:seg + size]
            for i in range(nn):
                codes = per_node.get(i, [])
                cat_off.append(len(cats))
                cat_len.append(len(codes))
                cats += codes
        arr = {
            "left": np.array(cols["left"], np.int32), "right": np.array(cols["right"], np.int32),
            "feat": np.array(cols["feat"], np.uint32), "value": np.array(cols["value"], np.float32),
            "dl": np.array(cols["dl"], np.uint8), "gain": np.array(cols["gain"], np.float32),
            "hess": np.array(cols["hess"], np.float32),
        }
        toff = np.array(off, np.uint32)
        coff = np.array(cat_off, np.uint64)
        clen = np.array(cat_len, np.uint32)
        carr = np.array(cats if cats else [0], np.uint32)
        h = self.lib.rc_model_load(len(trees), _ptr(toff, C.c_uint32), _ptr(arr["left"], C.c_int32),
                                   _ptr(arr["right"], C.c_int32), _ptr(arr["feat"], C.c_uint32),
                                   _ptr(arr["value"], C.c_float), _ptr(arr["dl"], C.c_uint8),
                                   _ptr(arr["gain"], C.c_float), _ptr(arr["hess"], C.c_float),
                                   _ptr(coff, C.c_uint64), _ptr(clen, C.c_uint32), _ptr(carr, C.c_uint32), nf,
                                   objective, base_score, _ptr(margins, C.c_float),
                                   num_class if margins is not None else 0, spw, _ptr(ftypes, C.c_uint8))
        if not h:
            raise ValueError(self.lib.rc_last_error().decode())
        return RefModel(self, h, nf)

    def softmax_gradients(self, margins, y, w=None):
        """margins K x n (class-major) -> K x n x 2 (g, h)."""
        m = np.ascontiguousarray(margins, dtype=np.float32)
        K, n = m.shape
        y = np.ascontiguousarray(y, dtype=np.float32)
        w = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
        out = np.zeros((K, n, 2), dtype=np.float32)
        self.lib.rc_softmax_gradients(_ptr(m, C.c_float), _ptr(y, C.c_float), _ptr(w, C.c_float), n, K,
                                      _ptr(out, C.c_float))
        return out

    def class_margins(self, y, K, w=None):
        y = np.ascontiguousarray(y, dtype=np.float32)
        w = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
        out = np.zeros(K, dtype=np.float32)
        self.lib.rc_class_margins(_ptr(y, C.c_float), _ptr(w, C.c_float), y.shape[0], K, _ptr(out, C.c_float))
        return out

    def last_timing(self):
        setup = C.c_double()
        rounds = (C.c_double * 100000)()
        k = self.lib.rc_last_timing(C.byref(setup), rounds, 100000)
        return setup.value, list(rounds[:k])

    # ---------------------------------------------------------------- components
    def sketch(self, X, max_bin, w=None, categorical=None, nthread=0):
        X = np.ascontiguousarray(X, dtype=np.float32)
        n, F = X.shape
        cap = F * (max(max_bin, 65536) + 1)
        cuts = np.zeros(cap, dtype=np.float32)
        off = np.zeros(F + 1, dtype=np.uint32)
        cat = None if categorical is None else np.ascontiguousarray(categorical, dtype=np.uint8)
        w = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
        k = self.lib.rc_sketch(_ptr(X, C.c_float), n, F, max_bin, _ptr(w, C.c_float), _ptr(cat, C.c_uint8),
                               _ptr(cuts, C.c_float), _ptr(off, C.c_uint32), cap, nthread)
        return cuts[:k].copy(), off

    def quantize(self, X, cuts, off, categorical=None):
        X = np.ascontiguousarray(X, dtype=np.float32)
        n, F = X.shape
        out = np.zeros((F, n), dtype=np.uint16)
        cat = None if categorical is None else np.ascontiguousarray(categorical, dtype=np.uint8)
        self.lib.rc_quantize(_ptr(X, C.c_float), n, F, _ptr(cuts, C.c_float), _ptr(off, C.c_uint32),
                             _ptr(cat, C.c_uint8), _ptr(out, C.c_uint16))
        return out

    def quantizer(self, gpair, n_rows=None):
        g = np.ascontiguousarray(gpair, dtype=np.float32)
        s = np.zeros(2, dtype=np.float64)
        rc = self.lib.rc_quantizer(_ptr(g, C.c_float), g.shape[0], n_rows or g.shape[0], _ptr(s, C.c_double))
        if rc:
            raise ValueError("non-finite gradient or Hessian")
        return s

    def pow2_scales(self, max_abs, n_rows):
        """types.rs:366-385 pow2_scale of each f32 bound."""
        v = np.ascontiguousarray(max_abs, dtype=np.float32)
        out = np.zeros(v.shape[0], dtype=np.float64)
        self.lib.rc_pow2_scales(_ptr(v, C.c_float), v.shape[0], n_rows, _ptr(out, C.c_double))
        return out

    def pow2_scale_digest(self, lo_bits, hi_bits, n_rows):
        """Digest of pow2_scale over the f32 bit patterns [lo_bits, hi_bits)."""
        return int(self.lib.rc_pow2_scale_digest(lo_bits, hi_bits, n_rows))

    def to_fixed(self, gpair, scales):
        g = np.ascontiguousarray(gpair, dtype=np.float32)
        out = np.zeros((g.shape[0], 2), dtype=np.int64)
        s = np.zeros(2, dtype=np.int64)
        sc = np.ascontiguousarray(scales, dtype=np.float64)
        self.lib.rc_to_fixed(_ptr(g, C.c_float), g.shape[0], _ptr(sc, C.c_double), _ptr(out, C.c_int64),
                             _ptr(s, C.c_int64))
        return out, s

    def hist(self, bins_colmajor, feat_offsets, missing, gpair_fixed, rows=None):
        b = np.ascontiguousarray(bins_colmajor, dtype=np.uint16)
        F, n = b.shape
        off = np.ascontiguousarray(feat_offsets, dtype=np.uint32)
        miss = np.ascontiguousarray(missing, dtype=np.uint16)
        g = np.ascontiguousarray(gpair_fixed, dtype=np.int64)
        out = np.zeros((int(off[-1]), 2), dtype=np.int64)
        r = None if rows is None else np.ascontiguousarray(rows, dtype=np.uint32)
        self.lib.rc_hist(_ptr(b, C.c_uint16), n, F, _ptr(off, C.c_uint32), _ptr(miss, C.c_uint16),
                         _ptr(g, C.c_int64), _ptr(r, C.c_uint32), 0 if r is None else r.shape[0],
                         _ptr(out, C.c_int64))
        return out

    def sample_features(self, nf, rate, seed, round_):
        out = np.zeros(max(nf, 1), dtype=np.uint32)
        k = self.lib.rc_sample_features(nf, rate, seed, round_, _ptr(out, C.c_uint32))
        return out[:k].copy()

    def rows_selected(self, n, rate, seed, tree):
        out = np.zeros(n, dtype=np.uint8)
        self.lib.rc_rows_selected(n, rate, seed, tree, _ptr(out, C.c_uint8))
        return out.astype(bool)

    def best_split(self, hist, feat_offsets, node_sum, scales, lower=-3.4028234663852886e38,
                   upper=3.4028234663852886e38, enabled=None, **kw):
        h = np.ascontiguousarray(hist, dtype=np.int64)
        off = np.ascontiguousarray(feat_offsets, dtype=np.uint32)
        ns = np.ascontiguousarray(node_sum, dtype=np.int64)
        sc = np.ascontiguousarray(scales, dtype=np.float64)
        en = None if enabled is None else np.ascontiguousarray(enabled, dtype=np.uint8)
        p = self.params(**kw)
        out = rc_split()
        self.lib.rc_best_split(_ptr(h, C.c_int64), off.shape[0] - 1, _ptr(off, C.c_uint32), _ptr(ns, C.c_int64),
                               _ptr(sc, C.c_double), C.byref(p), lower, upper, _ptr(en, C.c_uint8), C.byref(out))
        return out


class RefModel:
    def __init__(self, rc, handle, n_features):
        self.rc, self.h, self.n_features = rc, handle, n_features

    def __del__(self):
        try:
            self.rc.lib.rc_model_free(self.h)
        except Exception:
            pass

    @property
    def num_trees(self):
        return self.rc.lib.rc_model_num_trees(self.h)

    def json(self) -> bytes:
        n = self.rc.lib.rc_model_json(self.h, None, 0)
        buf = C.create_string_buffer(n)
        self.rc.lib.rc_model_json(self.h, buf, n)
        return buf.raw[:n]

    @property
    def num_outputs(self):
        return self.rc.lib.rc_model_num_outputs(self.h)

    def predict_margin(self, X, nthread=0):
        """Raw margins: n values, or n x num_class for a multiclass model."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        k = self.num_outputs
        out = np.zeros(X.shape[0] if k == 1 else (X.shape[0], k), dtype=np.float32)
        self.rc.lib.rc_predict_margin(self.h, _ptr(X, C.c_float), X.shape[0], _ptr(out, C.c_float), nthread)
        return out

    def shap(self, X, nthread=0):
        """n x (F+1), or n x K x (F+1) for a multiclass model."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        k = self.num_outputs
        out = np.zeros((X.shape[0], X.shape[1] + 1) if k == 1 else (X.shape[0], k, X.shape[1] + 1),
                       dtype=np.float32)
        self.rc.lib.rc_shap(self.h, _ptr(X, C.c_float), X.shape[0], _ptr(out, C.c_float), nthread)
        return out

    def pred_leaf(self, X, nthread=0):
        X = np.ascontiguousarray(X, dtype=np.float32)
        out = np.zeros((X.shape[0], self.num_trees), dtype=np.float32)
        self.rc.lib.rc_pred_leaf(self.h, _ptr(X, C.c_float), X.shape[0], _ptr(out, C.c_float), nthread)
        return out

    def approx_contribs(self, X, nthread=0):
        X = np.ascontiguousarray(X, dtype=np.float32)
        out = np.zeros((X.shape[0], X.shape[1] + 1), dtype=np.float32)
        self.rc.lib.rc_pred_approx(self.h, _ptr(X, C.c_float), X.shape[0], _ptr(out, C.c_float), nthread)
        return out

    def interactions(self, X, nthread=0):
        X = np.ascontiguousarray(X, dtype=np.float32)
        nc = X.shape[1] + 1
        out = np.zeros((X.shape[0], nc, nc), dtype=np.float32)
        self.rc.lib.rc_pred_interactions(self.h, _ptr(X, C.c_float), X.shape[0], _ptr(out, C.c_float), nthread)
        return out
