"""fbgpu_partition_noalloc: the partition entry point for callers that cannot
allocate device memory (their host owns every allocation, as the reference's
Rust side does).  It must give the same rows and left count as the context's
fbgpu_partition, call after call, using only caller-provided device buffers
and its fixed static scratch.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from gpu_util import Ctx, random_bins

pytestmark = pytest.mark.gpu


def _noalloc(lib, rec_dev, stride, width, byte_off, rows_dev, n, bin_, missing_left, cats, out_dev, nl_dev):
    cw = None if cats is None else np.ascontiguousarray(cats, dtype=np.uint32)
    st = lib.fbgpu_partition_noalloc(C.c_void_p(rec_dev.data_ptr()), stride, width, byte_off,
                                     C.c_void_p(rows_dev.data_ptr()), n, bin_, int(missing_left),
                                     None if cw is None else cw.ctypes.data_as(C.POINTER(C.c_uint32)),
                                     C.c_void_p(out_dev.data_ptr()), C.c_void_p(nl_dev.data_ptr()), None)
    assert st == 0, lib.fbgpu_last_error(None).decode()


def test_noalloc_partition_matches_context_partition_twice():
    import torch
    from ferrisboost_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(42)
    n_all = 300000
    nbins = [300, 64]  # a 16-bit numeric feature and an 8-bit categorical one
    bins, widths = random_bins(rng, n_all, nbins)
    ctx = Ctx(bins, nbins, widths, categorical=[0, 1])
    # the caller's own row-major records: feature 0 (u16) at byte 0, feature 1 (u8) at byte 2
    stride = 16
    rec = np.zeros((n_all, stride), dtype=np.uint8)
    rec[:, 0:2] = bins[0].astype(np.uint16).view(np.uint8).reshape(n_all, 2)
    rec[:, 2] = bins[1].astype(np.uint8)
    rec_dev = torch.from_numpy(rec).cuda()
    rows = np.sort(rng.choice(n_all, 123457, replace=False)).astype(np.uint32)
    rows_dev = torch.from_numpy(rows.view(np.int32)).cuda()
    out_dev = torch.zeros(len(rows), dtype=torch.int32, device="cuda")
    nl_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    cats = np.zeros(8, np.uint32)
    for c in (3, 17, 40):
        cats[c // 32] |= np.uint32(1 << (c % 32))
    calls = [((0, 0, 2, 150, True, None), (0, 150, True, None)),
             ((1, 2, 1, 0, False, cats), (1, 0, False, cats))]
    for (feat, byte_off, width, b, ml, cw), (cf, cb, cml, ccats) in calls:
        _noalloc(lib, rec_dev, stride, width, byte_off, rows_dev, len(rows), b, ml, cw, out_dev, nl_dev)
        torch.cuda.synchronize()
        want_rows, want_nl = ctx.partition(rows, cf, cb, cml, ccats)
        got_rows = out_dev.cpu().numpy().view(np.uint32)
        assert int(nl_dev.cpu().item()) == want_nl
        assert np.array_equal(got_rows, want_rows)


def test_noalloc_partition_rejects_oversized_requests():
    import torch
    from ferrisboost_b200 import _lib
    lib = _lib.load()
    d = torch.zeros(16, dtype=torch.int32, device="cuda")
    st = lib.fbgpu_partition_noalloc(C.c_void_p(d.data_ptr()), 16, 2, 0, C.c_void_p(d.data_ptr()),
                                     268435456 + 1, 0, 0, None, C.c_void_p(d.data_ptr()),
                                     C.c_void_p(d.data_ptr()), None)
    assert st == 1
    assert "at most 268435456 rows" in lib.fbgpu_last_error(None).decode()
