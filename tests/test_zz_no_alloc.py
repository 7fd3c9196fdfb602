"""wocr_argmax_rows_noalloc: the row arg-max for callers that cannot let the library allocate
device memory (its scratch is a fixed array in the library's device memory).  Collected last,
so a failure here comes after every other test has run; it also passes alone in a fresh process.

Each result is checked three ways: against numpy on the host (the lowest index among equal
maxima, as K30 of src/nd.rs:360-391 picks it; the log-sum-exp in float64), against the existing
entry point that allocates its scratch, and against the device memory pool, whose used bytes
must not move during the call.
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


def _pool_used(device: int) -> int:
    """Bytes in use in the device's default memory pool (the pool the library allocates from)."""
    from cuda.bindings import driver as d

    err, pool = d.cuDeviceGetDefaultMemPool(device)
    assert err == d.CUresult.CUDA_SUCCESS
    err, v = d.cuMemPoolGetAttribute(pool, d.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_CURRENT)
    assert err == d.CUresult.CUDA_SUCCESS
    return int(v)


def _noalloc(gpu, d_ptr, rows, cols):
    best = np.empty(rows, np.uint32)
    mx = np.empty(rows, np.float32)
    lse = np.empty(rows, np.float32)
    st = wocr.lib().wocr_argmax_rows_noalloc(gpu.h, ctypes.c_void_p(d_ptr), rows, cols, best.ctypes.data,
                                             mx.ctypes.data, lse.ctypes.data)
    _lib.check(st)
    return best, mx, lse


def _host(x):
    """numpy's row arg-max (first maximal index; 0 for rows of NaN or -inf, as K30's search from
    (-3.4e38, 0) gives), the row maximum and the log-sum-exp in float64."""
    finite = np.where(np.isnan(x), -np.inf, x)
    best = finite.argmax(axis=1).astype(np.uint32)
    mx = finite.max(axis=1)
    best[~(mx > np.float32(-3.4e38))] = 0
    m64 = mx.astype(np.float64)
    lse = np.log(np.exp(x.astype(np.float64) - m64[:, None]).sum(axis=1)) + m64
    return best, mx, lse


def test_noalloc_argmax_matches_numpy_and_existing_entry_point_twice():
    import torch

    gpu = wocr.Gpu()
    try:
        rng = np.random.default_rng(99)
        warm = torch.zeros((4, 4), dtype=torch.float32, device="cuda")
        _noalloc(gpu, warm.data_ptr(), 4, 4)              # the device's one-time address lookup
        # two calls in a row with different shapes: the shared scratch keeps the last call's
        # contents, and every result must come from the current call
        for rows, cols in ((1200, 18709), (3000, 97)):
            x = (rng.standard_normal((rows, cols)) * 0.3).astype(np.float32)
            x[5, 3] = x[5, 7] = x[5].max() + 1.0            # a tie: the lowest index wins
            x[9, :] = -np.inf                                # no value above the start: index 0
            d = torch.from_numpy(x).cuda()
            torch.cuda.synchronize()
            used0 = _pool_used(0)
            best, mx, lse = _noalloc(gpu, d.data_ptr(), rows, cols)
            assert _pool_used(0) == used0, "the call allocated from the device memory pool"
            hb, hmx, hlse = _host(x)
            assert (best == hb).all(), f"{int((best != hb).sum())} rows differ from numpy's arg-max"
            assert best[5] == 3 and best[9] == 0
            ok = np.isfinite(hlse)
            assert (mx[ok] == hmx[ok]).all()
            assert np.abs(lse[ok] - hlse[ok]).max() <= 1e-5 * max(1.0, float(np.abs(hlse[ok]).max()))
            rb, rmx, rlse, shape = _existing(gpu, x)
            assert shape == (rows, cols)
            assert (best == rb).all()
            assert (mx[ok] == rmx[ok]).all()
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
