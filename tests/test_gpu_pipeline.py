"""Record-then-read (`wocr_batch`, the reference's encoder + Gpu::read_many) and the multi-page
PP-OCRv6 pipeline (`wocr_pp_pages`: lanes and merged recognitions, src/bin/ocr-bench.rs:133-310,
458-585).  Merging and lanes change when work runs, never what it computes: every result must
equal the page-at-a-time and call-at-a-time results exactly."""
import numpy as np
import pytest

import wocr
from wocr import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pp_rec():
    return synth.pp_rec_model()


def test_argmax_enqueue_equals_synchronous_calls(gpu, pp_rec):
    """Several batches recorded with one wait, including the same shape three times in a row (a
    direct first run, the capture, a replay) with different data: each result equals the
    synchronous call's on the same input."""
    lines = synth.pp_lines(5, n=40)
    batches, _ = synth.pp_batches(lines)
    same = [b for b in batches if b[2] == batches[0][2]][:1] * 3
    rng = np.random.default_rng(1)
    inputs = [d for d, _, _ in batches[:3]] + [np.clip(d + rng.standard_normal(d.shape).astype(np.float32) * 0.1, -1, 1)
                                               for d, _, _ in same]
    g = wocr.NdGraph(gpu, pp_rec, stop_before_softmax=True)
    h = wocr.NdGraph(gpu, pp_rec, stop_before_softmax=True)
    try:
        with wocr.Batch(gpu) as b:
            pend = [g.argmax_enqueue(b, x) for x in inputs]
            assert b.pending == len(inputs)
            assert not any(p.done for p in pend)
            b.wait()
            assert b.pending == 0
            for x, p in zip(inputs, pend):
                assert p.done
                best, mx, lse, shape = h.argmax(x)
                assert p.shape == shape
                np.testing.assert_array_equal(p.best, best)
                np.testing.assert_array_equal(p.row_max, mx)
                np.testing.assert_array_equal(p.row_lse, lse)
            # the batch is reusable after a wait
            p2 = g.argmax_enqueue(b, inputs[0])
            b.wait(timeout_ms=60000)
            np.testing.assert_array_equal(p2.best, pend[0].best)
    finally:
        g.close()
        h.close()


def test_batch_of_another_context_is_rejected(gpu, pp_rec):
    other = wocr.Gpu(lines=8, device=0)
    g = wocr.NdGraph(gpu, pp_rec, stop_before_softmax=True)
    try:
        with wocr.Batch(other) as b:
            with pytest.raises(wocr.WocrError) as e:
                g.argmax_enqueue(b, np.zeros((1, 3, 48, 64), np.float32))
            assert e.value.code == 1
            b.wait()  # nothing recorded: returns at once
    finally:
        g.close()
        other.close()


def _pages(n, w=1275, h=1650, bands=10, seed=40):
    return [synth.page(seed + k, w, h, bands=bands) for k in range(n)]


@pytest.mark.parametrize("merge,lanes", [(1, 1), (3, 1), (2, 2), (1, 3)])
def test_pp_pages_equal_page_by_page(gpu, pp_rec, merge, lanes):
    """Five pages with an ink detector (dozens of lines each) through wocr_pp_pages: boxes and
    every line's classes equal wocr_pp_page's, page by page."""
    pages = _pages(5)
    with wocr.PPPipeline(gpu, synth.pp_ink_det_model(), pp_rec) as pp:
        want = [pp.page(pg, 1275, 1650) for pg in pages]
        got = pp.pages(pages, 1275, 1650, merge=merge, lanes=lanes)
        assert pp.last_bytes[0] == 5 * 1275 * 1650 * 3
    assert sum(len(b) for b, _ in want) >= 200
    for (wb, wl), (gb, gl) in zip(want, got):
        np.testing.assert_array_equal(gb, wb)
        assert len(gl) == len(wl)
        for a, c in zip(gl, wl):
            np.testing.assert_array_equal(a, c)


def test_pp_pages_from_device_memory_and_boxes_only(gpu, pp_rec):
    import torch

    pages = _pages(3, seed=60)
    d = [torch.from_numpy(p).cuda() for p in pages]
    torch.cuda.synchronize()
    with wocr.PPPipeline(gpu, synth.pp_ink_det_model(), pp_rec) as pp:
        host = pp.pages(pages, 1275, 1650, merge=2, lanes=2)
        dev = pp.pages([t.data_ptr() for t in d], 1275, 1650, merge=2, lanes=2)
        assert pp.last_bytes[0] == 0            # nothing crossed PCIe for the pages
        only = pp.pages(pages, 1275, 1650, lanes=2, boxes_only=True)
    for (hb, hl), (db, dl), (ob, ol) in zip(host, dev, only):
        np.testing.assert_array_equal(db, hb)
        np.testing.assert_array_equal(ob, hb)
        assert ol == []
        for a, c in zip(dl, hl):
            np.testing.assert_array_equal(a, c)


def test_pp_pages_full_size_random_detector(gpu, pp_rec):
    """Config 4 as specified (random-init DB detector, 2550 x 3300 pages) over 3 lanes."""
    pages = [synth.page(3000 + k, 2550, 3300) for k in range(4)]
    with wocr.PPPipeline(gpu, synth.pp_det_model(), pp_rec) as pp:
        want = [pp.page(pg, 2550, 3300) for pg in pages]
        got = pp.pages(pages, 2550, 3300, merge=2, lanes=3)
    for (wb, wl), (gb, gl) in zip(want, got):
        np.testing.assert_array_equal(gb, wb)
        for a, c in zip(gl, wl):
            np.testing.assert_array_equal(a, c)
