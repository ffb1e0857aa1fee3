"""Helpers for the GPU parity tests: a training context driven through the C ABI."""
import ctypes as C

import numpy as np

from ferrisboost_b200 import _lib


def lib():
    return _lib.load()


def check(status, ctx=None):
    if status != 0:
        msg = lib().fbgpu_last_error(ctx).decode()
        raise RuntimeError(f"fbgpu status {status}: {msg}")


class Ctx:
    """fbgpu_ctx over column-major bins (F x n uint16; missing 255 / 65535)."""

    def __init__(self, bins, nbins, widths, categorical=None, max_depth=6, max_leaves=0, device=0):
        bins = np.ascontiguousarray(bins, dtype=np.uint16)
        F, n = bins.shape
        self.F, self.n = F, n
        cfg = _lib.FbgpuConfig(device=device, n_features=F, n_rows=n, n_rows_global=n, row_offset=0,
                               max_depth=max_depth, max_leaves=max_leaves, hist_smem_bytes=0, gpu_math=0)
        h = C.c_void_p()
        check(lib().fbgpu_ctx_create(C.byref(cfg), C.byref(h)))
        self.h = h
        nb = np.ascontiguousarray(nbins, dtype=np.uint32)
        w = np.ascontiguousarray(widths, dtype=np.uint8)
        cat = None if categorical is None else np.ascontiguousarray(categorical, dtype=np.uint8)
        check(lib().fbgpu_set_features(h, _lib.ptr(nb, C.c_uint32), _lib.ptr(w, C.c_uint8),
                                       _lib.ptr(cat, C.c_uint8)), h)
        for width in (1, 2):
            feats = [f for f in range(F) if w[f] == width]
            per = 64 if width == 2 else 128
            for i in range(0, len(feats), per):
                ids = np.array(feats[i:i + per], dtype=np.uint32)
                data = np.ascontiguousarray(bins[ids].astype(np.uint16 if width == 2 else np.uint8))
                check(lib().fbgpu_upload_block(h, _lib.ptr(ids, C.c_uint32), len(ids), width,
                                               data.ctypes.data_as(C.c_void_p)), h)
        self.hoff = np.concatenate([[0], np.cumsum(nb)]).astype(np.uint32)

    def __del__(self):
        if getattr(self, "h", None):
            lib().fbgpu_ctx_destroy(self.h)
            self.h = None

    def histogram(self, fixed, rows=None):
        fixed = np.ascontiguousarray(fixed, dtype=np.int64)
        out = np.zeros((int(self.hoff[-1]), 2), dtype=np.int64)
        r = None if rows is None else np.ascontiguousarray(rows, dtype=np.uint32)
        check(lib().fbgpu_histogram(self.h, _lib.ptr(r, C.c_uint32), 0 if r is None else len(r),
                                    _lib.ptr(fixed, C.c_int64), _lib.ptr(out, C.c_int64)), self.h)
        return out

    def eval_split(self, hist, node_sum, scales, lower=-3.4028234663852886e38, upper=3.4028234663852886e38,
                   enabled=None, monotone=None, **kw):
        tp = _lib.FbgpuTreeParams(eta=kw.get("eta", 0.3), reg_lambda=kw.get("reg_lambda", 1.0),
                                  gamma=kw.get("gamma", 0.0), min_child_weight=kw.get("min_child_weight", 1.0),
                                  alpha=kw.get("alpha", 0.0), max_delta_step=kw.get("max_delta_step", 0.0),
                                  max_depth=6, max_leaves=0, max_cat_to_onehot=kw.get("max_cat_to_onehot", 4),
                                  max_cat_threshold=kw.get("max_cat_threshold", 64), grow_policy=0)
        mono = None
        if monotone is not None:
            mono = np.ascontiguousarray(monotone, dtype=np.int8)
            tp.monotone = _lib.ptr(mono, C.c_int8)
        h = np.ascontiguousarray(hist, dtype=np.int64)
        ns = np.ascontiguousarray(node_sum, dtype=np.int64)
        sc = np.ascontiguousarray(scales, dtype=np.float64)
        en = None if enabled is None else np.ascontiguousarray(enabled, dtype=np.uint8)
        out = _lib.FbgpuSplit()
        check(lib().fbgpu_eval_split(self.h, _lib.ptr(h, C.c_int64), _lib.ptr(ns, C.c_int64),
                                     _lib.ptr(sc, C.c_double), C.byref(tp), lower, upper, _lib.ptr(en, C.c_uint8),
                                     C.byref(out)), self.h)
        return out

    def partition(self, rows, feat, bin_, missing_left, cats=None):
        rows = np.ascontiguousarray(rows, dtype=np.uint32)
        out = np.zeros_like(rows)
        nl = C.c_uint64()
        cw = None if cats is None else np.ascontiguousarray(cats, dtype=np.uint32)
        check(lib().fbgpu_partition(self.h, _lib.ptr(rows, C.c_uint32), len(rows), feat, bin_, int(missing_left),
                                    _lib.ptr(cw, C.c_uint32), _lib.ptr(out, C.c_uint32), C.byref(nl)), self.h)
        return out, nl.value


    def cat_words(self):
        return lib().fbgpu_ctx_cat_words(self.h)

    def partition_set(self, rows, feat, missing_left, words):
        rows = np.ascontiguousarray(rows, dtype=np.uint32)
        out = np.zeros_like(rows)
        nl = C.c_uint64()
        cw = np.ascontiguousarray(words, dtype=np.uint32)
        check(lib().fbgpu_partition_set(self.h, _lib.ptr(rows, C.c_uint32), len(rows), feat, int(missing_left),
                                        _lib.ptr(cw, C.c_uint32), len(cw), _lib.ptr(out, C.c_uint32),
                                        C.byref(nl)), self.h)
        return out, nl.value


def random_bins(rng, n, nbins, miss_rate=0.05):
    """Column-major random bins with per-width missing sentinels."""
    F = len(nbins)
    widths = np.array([2 if nb > 255 else 1 for nb in nbins], dtype=np.uint8)
    bins = np.zeros((F, n), dtype=np.uint16)
    for f, nb in enumerate(nbins):
        bins[f] = rng.integers(0, nb, n)
        miss = 65535 if widths[f] == 2 else 255
        bins[f][rng.random(n) < miss_rate] = miss
    return bins, widths
