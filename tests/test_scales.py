"""Quantizer scales.  Exact-mode training computes each round's power-of-two
scales on the device: the binary exponent of raw = (2^62 / n_rows) / max_abs,
except for the f32 bounds the host lists for the row count, where the
reference's floor(log2(raw)) with the host's log2 differs
(ferrisboost_b200/csrc/qscale.h).  These tests compare that rule with the
oracle's restatement of the reference's pow2_scale (src/types.rs:366-385):
on every positive finite f32 by a digest, densely around every power-of-two
boundary for several row counts, and on the GPU."""
import ctypes as C

import numpy as np
import pytest

import ferrisboost_b200 as fb
from ferrisboost_b200 import _lib

POSITIVE_FINITE = (1, 0x7F800000)  # f32 bit patterns of (0, +inf)


def _scales(values, n_rows, device=-1):
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.zeros(v.shape[0], dtype=np.float64)
    st = fb.lib().fbgpu_quantizer_scales(device, _lib.ptr(v, C.c_float), v.shape[0], n_rows,
                                         _lib.ptr(out, C.c_double))
    assert st == 0, fb.lib().fbgpu_last_error(None)
    return out


def _near_boundaries(n_rows, span=48):
    """Every f32 within `span` ulps of budget / 2^k for all k (raw within a few
    ulps of each power of two), plus special values."""
    budget = float(2**62) / float(max(n_rows, 1))
    centers = []
    for k in range(-1100, 1100):
        t = np.ldexp(budget, -k)
        if 0.0 < t < 3.4e38:
            c = np.float32(t)
            if c > 0:
                centers.append(c.view(np.uint32))
    centers = np.unique(np.array(centers, dtype=np.int64))
    offs = np.arange(-span, span + 1, dtype=np.int64)
    bits = (centers[:, None] + offs[None, :]).ravel()
    bits = bits[(bits >= POSITIVE_FINITE[0]) & (bits < POSITIVE_FINITE[1])]
    v = np.unique(bits).astype(np.uint32).view(np.float32)
    special = np.array([0.0, -0.0, -1.0, np.inf, -np.inf, np.nan, 1e-45, 1.17549435e-38,
                        3.4028235e38, 1.0, 0.25, 0.5], dtype=np.float32)
    return np.concatenate([v, special])


@pytest.mark.parametrize("n_rows", [11_000_000, 3])
def test_scale_digest_over_every_positive_f32(oracle, n_rows):
    lo, hi = POSITIVE_FINITE
    got = int(fb.lib().fbgpu_quantizer_scale_digest(lo, hi, n_rows))
    want = oracle.pow2_scale_digest(lo, hi, n_rows)
    assert got == want


@pytest.mark.parametrize("n_rows", [0, 1, 2, 3, 1000, 30_001, 1_000_000, 11_000_000, 2**40 + 17, 2**64 - 1])
def test_scales_around_every_power_of_two(oracle, n_rows):
    v = _near_boundaries(n_rows)
    got = _scales(v, n_rows)
    want = oracle.pow2_scales(v, n_rows)
    bad = np.nonzero(got.view(np.uint64) != want.view(np.uint64))[0]
    assert bad.size == 0, [(float(v[i]), got[i], want[i]) for i in bad[:5]]


def test_scale_digest_sums_its_parts_and_sees_one_value(oracle):
    # the digest of a range is the sum of its parts (a mismatch can be
    # bisected), and one differing scale changes it
    n = 11_000_000
    lo = int(np.float32(0.5).view(np.uint32))
    whole = oracle.pow2_scale_digest(lo, lo + 1000, n)
    parts = (oracle.pow2_scale_digest(lo, lo + 999, n) + oracle.pow2_scale_digest(lo + 999, lo + 1000, n)) % 2**64
    assert whole == parts
    assert int(fb.lib().fbgpu_quantizer_scale_digest(lo, lo + 1000, n)) == whole
    one = oracle.pow2_scale_digest(lo + 999, lo + 1000, n)
    other = oracle.pow2_scale_digest(lo + 999, lo + 1000, 2 * n)  # the same f32, half the scale
    assert one != other


@pytest.mark.gpu
@pytest.mark.parametrize("n_rows", [3, 1_000_000, 11_000_000])
def test_device_scales_equal_reference(oracle, n_rows):
    rng = np.random.default_rng(n_rows % 1000)
    rand = rng.integers(POSITIVE_FINITE[0], POSITIVE_FINITE[1], 2_000_000, dtype=np.uint32).view(np.float32)
    v = np.concatenate([_near_boundaries(n_rows), rand])
    got = _scales(v, n_rows, device=0)
    want = oracle.pow2_scales(v, n_rows)
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
