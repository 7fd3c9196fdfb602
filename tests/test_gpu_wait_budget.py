"""The bounded waits of the tensor-core GEMM on the device (the failure path of its mbarrier
waits): with a short clock budget and a first A stage whose producers never arrive, the MMA
thread's wait runs out; the kernel records its error code, drains, frees its tensor memory and
returns, the host reports WOCR_ERR_TIMEOUT, and the same context then runs the graph again with
the results of a clean run.  No fault and no hang: every other wait of the kernel ends on the
abort flag or on the same budget."""
import numpy as np
import pytest

import wocr
from wocr.synth import _Builder

pytestmark = pytest.mark.gpu

WOCR_ERR_TIMEOUT = 6


def test_umma_wait_runs_out_and_context_stays_usable(gpu, monkeypatch):
    b = _Builder(21)
    y = b.linear("x", 120, 97)
    g = wocr.NdGraph(gpu, b.model("x", y))
    x = np.random.default_rng(4).standard_normal((1, 40, 120)).astype(np.float32)
    try:
        clean = g.run(x)
        monkeypatch.setenv("WOCR_NO_GRAPH", "1")
        monkeypatch.setenv("WOCR_WAIT_BUDGET", "2000000")  # clock cycles, about 1 ms
        monkeypatch.setenv("WOCR_TEST_STALL_FIRST_STAGE", "1")
        with pytest.raises(wocr.WocrError) as err:
            g.run(x)
        assert err.value.code == WOCR_ERR_TIMEOUT, err.value
        assert "wait gave up" in str(err.value)
        monkeypatch.delenv("WOCR_TEST_STALL_FIRST_STAGE")
        # the same context, eager and then replayed from a graph: the clean results
        again = g.run(x)
        assert np.array_equal(again, clean)
        monkeypatch.delenv("WOCR_WAIT_BUDGET")
        monkeypatch.delenv("WOCR_NO_GRAPH")
        assert np.array_equal(g.run(x), clean)
    finally:
        g.close()
