"""The device reproduction of the host libm expf (exact-mode logistic
gradients, objective.rs:37-39 of the reference) equals the host's expf on
every one of the 2^32 f32 inputs, and exact training falls back to host exp
values when asked to."""
import ctypes as C
import os

import numpy as np
import pytest

import ferrisboost_b200 as fb
from ferrisboost_b200 import _lib

pytestmark = pytest.mark.gpu


def test_device_expf_equals_host_expf_on_every_input():
    lib = _lib.load()
    chunk = 1 << 28
    total = 0
    reports = []
    for begin in range(0, 1 << 32, chunk):
        bad = C.c_uint64()
        rep = np.zeros(16, np.uint32)
        assert lib.fbgpu_expf_check(0, begin, chunk, C.byref(bad), _lib.ptr(rep, C.c_uint32)) == 0, \
            lib.fbgpu_last_error(None)
        total += bad.value
        if bad.value:
            reports.append(rep.reshape(4, 4)[: min(4, bad.value)])
    assert total == 0, [[hex(int(v)) for v in r] for rep in reports for r in rep]


def test_exact_logistic_host_and_device_exp_give_the_same_model(oracle, monkeypatch):
    rng = np.random.default_rng(8)
    X = rng.standard_normal((20000, 10)).astype(np.float32)
    y = (rng.random(20000) < 1 / (1 + np.exp(-X[:, 0] * 3))).astype(np.float32)
    p = {"objective": "binary:logistic", "max_depth": 6, "eta": 0.5, "max_bin": 256}
    dev = fb.train(p, X, label=y, num_boost_round=10).to_json()
    monkeypatch.setenv("FBGPU_EXACT_EXP", "host")
    host = fb.train(p, X, label=y, num_boost_round=10).to_json()
    assert dev == host == oracle.train(X, y, n_rounds=10, **p).json()
