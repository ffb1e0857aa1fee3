"""fbgpu_partition_noalloc: the partition entry point for callers that cannot
allocate device memory (their host owns every allocation, as the reference's
Rust side does).  It must give the same rows and left count as the context's
fbgpu_partition, call after call, using only caller-provided device buffers
and its fixed static scratch, and it must not allocate.  This file is
collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from gpu_util import Ctx, random_bins

pytestmark = pytest.mark.gpu

NO_MISSING = 0xFFFFFFFF


def _call(lib, rec_dev, stride, width, byte_off, missing, rows_dev, n, bin_, missing_left, cats, out_dev, nl_dev,
          stream=None, rec_offset=0):
    cw = None if cats is None else np.ascontiguousarray(cats, dtype=np.uint32)
    return lib.fbgpu_partition_noalloc(C.c_void_p(rec_dev.data_ptr() + rec_offset), stride, width, byte_off, missing,
                                       C.c_void_p(rows_dev.data_ptr()), n, bin_, int(missing_left),
                                       None if cw is None else cw.ctypes.data_as(C.POINTER(C.c_uint32)),
                                       C.c_void_p(out_dev.data_ptr()), C.c_void_p(nl_dev.data_ptr()), stream)


def _noalloc(lib, *args, **kw):
    st = _call(lib, *args, **kw)
    assert st == 0, lib.fbgpu_last_error(None).decode()


def _setup(rng, n_all=300000, n_rows=123457):
    import torch
    nbins = [300, 64]  # a 16-bit numeric feature and an 8-bit categorical one
    bins, widths = random_bins(rng, n_all, nbins)
    ctx = Ctx(bins, nbins, widths, categorical=[0, 1])
    # the caller's own row-major records: feature 0 (u16) at byte 0, feature 1 (u8) at byte 2
    stride = 16
    rec = np.zeros((n_all, stride), dtype=np.uint8)
    rec[:, 0:2] = bins[0].astype(np.uint16).view(np.uint8).reshape(n_all, 2)
    rec[:, 2] = bins[1].astype(np.uint8)
    rec_dev = torch.from_numpy(rec).cuda()
    rows = np.sort(rng.choice(n_all, n_rows, replace=False)).astype(np.uint32)
    rows_dev = torch.from_numpy(rows.view(np.int32)).cuda()
    out_dev = torch.zeros(len(rows), dtype=torch.int32, device="cuda")
    nl_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    return ctx, bins, rec, rec_dev, rows, rows_dev, out_dev, nl_dev, stride


def test_noalloc_partition_matches_context_partition_twice():
    import torch
    from ferrisboost_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(42)
    ctx, _, _, rec_dev, rows, rows_dev, out_dev, nl_dev, stride = _setup(rng)
    cats = np.zeros(8, np.uint32)
    for c in (3, 17, 40):
        cats[c // 32] |= np.uint32(1 << (c % 32))
    calls = [((0, 0, 2, 65535, 150, True, None), (0, 150, True, None)),
             ((1, 2, 1, 255, 0, False, cats), (1, 0, False, cats))]
    for (feat, byte_off, width, miss, b, ml, cw), (cf, cb, cml, ccats) in calls:
        _noalloc(lib, rec_dev, stride, width, byte_off, miss, rows_dev, len(rows), b, ml, cw, out_dev, nl_dev)
        torch.cuda.synchronize()
        want_rows, want_nl = ctx.partition(rows, cf, cb, cml, ccats)
        got_rows = out_dev.cpu().numpy().view(np.uint32)
        assert int(nl_dev.cpu().item()) == want_nl
        assert np.array_equal(got_rows, want_rows)


def test_noalloc_partition_allocates_nothing_and_runs_on_a_side_stream():
    import torch
    from ferrisboost_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(7)
    ctx, _, _, rec_dev, rows, rows_dev, out_dev, nl_dev, stride = _setup(rng)
    splits = (20, 150, 290)
    outs = [torch.zeros(len(rows), dtype=torch.int32, device="cuda") for _ in splits]
    nls = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in splits]
    side = torch.cuda.Stream()
    # the first call on this device resolves the scratch array's address
    _noalloc(lib, rec_dev, stride, 2, 0, 65535, rows_dev, len(rows), 100, False, None, out_dev, nl_dev)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for b, o, nl in zip(splits, outs, nls):
        _noalloc(lib, rec_dev, stride, 2, 0, 65535, rows_dev, len(rows), b, True, None, o, nl,
                 stream=C.c_void_p(side.cuda_stream))
    side.synchronize()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    for b, o, nl in zip(splits, outs, nls):
        want_rows, want_nl = ctx.partition(rows, 0, b, True, None)
        assert int(nl.cpu().item()) == want_nl
        assert np.array_equal(o.cpu().numpy().view(np.uint32), want_rows)


def test_noalloc_partition_full_range_one_byte_bins():
    # a 256-bin feature stored in one byte has no missing sentinel: bin 255
    # is an ordinary bin and compares with the split bin
    import torch
    from ferrisboost_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(3)
    n = 50000
    b = rng.integers(0, 256, n).astype(np.uint8)
    b[:1000] = 255
    rec = np.zeros((n, 16), np.uint8)
    rec[:, 5] = b
    rec_dev = torch.from_numpy(rec).cuda()
    rows = np.arange(0, n, 2, dtype=np.uint32)
    rows_dev = torch.from_numpy(rows.view(np.int32)).cuda()
    out_dev = torch.zeros(len(rows), dtype=torch.int32, device="cuda")
    nl_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    for split_bin, ml in ((200, True), (256, False)):
        _noalloc(lib, rec_dev, 16, 1, 5, NO_MISSING, rows_dev, len(rows), split_bin, ml, None, out_dev, nl_dev)
        torch.cuda.synchronize()
        left = b[rows] < split_bin
        want = np.concatenate([rows[left], rows[~left]])
        assert int(nl_dev.cpu().item()) == int(left.sum())
        assert np.array_equal(out_dev.cpu().numpy().view(np.uint32), want)


def test_noalloc_partition_rejects_invalid_requests():
    import torch
    from ferrisboost_b200 import _lib
    lib = _lib.load()
    d = torch.zeros(1024, dtype=torch.int32, device="cuda")
    o = torch.zeros(1024, dtype=torch.int32, device="cuda")
    nl = torch.zeros(4, dtype=torch.int32, device="cuda")

    def err(**kw):
        args = dict(stride=16, width=2, byte_off=0, missing=65535, n=100, out=o, rec_offset=0)
        args.update(kw)
        st = _call(lib, d, args["stride"], args["width"], args["byte_off"], args["missing"], d, args["n"], 0, 0,
                   None, args["out"], nl, rec_offset=args["rec_offset"])
        return st, lib.fbgpu_last_error(None).decode()

    st, msg = err(n=268435456 + 1)
    assert st == 1 and "at most 268435456 rows" in msg
    for kw in ({"stride": 15}, {"byte_off": 1}, {"rec_offset": 1}):
        st, msg = err(**kw)
        assert st == 1 and "two-byte bins need an even" in msg, kw
    st, msg = err(out=d)
    assert st == 1 and "must not overlap" in msg
    st, msg = err(width=1, byte_off=16)
    assert st == 1 and "outside the row record" in msg
