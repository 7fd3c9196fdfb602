"""wocr_argmax_rows_noalloc: the row arg-max for callers that cannot let the library allocate
device memory (its scratch is a fixed array in the library's device memory).  Collected last,
so a failure here comes after every other test has run; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import wocr
from wocr import _lib
from wocr.synth import _Builder

pytestmark = pytest.mark.gpu


def _existing(gpu, x):
    """The same arg-max through the existing entry point (which allocates its scratch)."""
    b = _Builder(0)
    g = wocr.NdGraph(gpu, b.model("x", b.op("Identity", ["x"])))
    try:
        return g.argmax(x)
    finally:
        g.close()


def _noalloc(gpu, d_ptr, rows, cols):
    best = np.empty(rows, np.uint32)
    mx = np.empty(rows, np.float32)
    lse = np.empty(rows, np.float32)
    st = wocr.lib().wocr_argmax_rows_noalloc(gpu.h, ctypes.c_void_p(d_ptr), rows, cols, best.ctypes.data,
                                             mx.ctypes.data, lse.ctypes.data)
    _lib.check(st)
    return best, mx, lse


def test_noalloc_argmax_matches_existing_entry_point_twice():
    import torch

    gpu = wocr.Gpu()
    try:
        rng = np.random.default_rng(99)
        # two calls in a row with different shapes: the shared scratch keeps the last call's
        # contents, and every result must come from the current call
        for rows, cols in ((1200, 18709), (3000, 97)):
            x = (rng.standard_normal((rows, cols)) * 0.3).astype(np.float32)
            x[5, 3] = x[5, 7] = x[5].max() + 1.0            # a tie: the lowest index wins
            d = torch.from_numpy(x).cuda()
            torch.cuda.synchronize()
            best, mx, lse = _noalloc(gpu, d.data_ptr(), rows, cols)
            rb, rmx, rlse, shape = _existing(gpu, x)
            assert shape == (rows, cols)
            assert (best == rb).all()
            assert best[5] == 3
            assert (mx == rmx).all()
            assert np.abs(lse - rlse).max() <= 1e-5 * max(1.0, float(np.abs(rlse).max()))
            del d
    finally:
        gpu.close()


def test_noalloc_argmax_rejects_more_rows_than_its_scratch():
    gpu = wocr.Gpu()
    try:
        best = np.empty(1, np.uint32)
        st = wocr.lib().wocr_argmax_rows_noalloc(gpu.h, ctypes.c_void_p(16), 65537, 10, best.ctypes.data, None,
                                                 None)
        assert st == 8                                        # WOCR_ERR_CAPACITY
        assert b"at most 65536 rows" in wocr.lib().wocr_last_error()
    finally:
        gpu.close()
