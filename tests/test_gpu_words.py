"""Word rectangles of detection masks on the device (`wocr_word_rects`, src/bin/ocr-bench.rs:
38-60) against the C restatement (`oracle_word_rects`): bit-identical rectangles, in the same
order, for nested shapes, edge shapes, noise, random blobs, empty and full masks, several pages
in one call, masks already on the device, and a config 1 detection mask."""
import numpy as np
import pytest

import wocr
from oracle import ref
from wocr import synth

from _helpers import pack_bits, word_masks

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k", range(5))
@pytest.mark.parametrize("params", [(3.0, 0.0, 100.0), (0.0, 0.0, 0.0), (3.0, 2.0, 50.0)])
def test_word_rects_bit_exact(gpu, k, params):
    m = word_masks()[k]
    h, w = m.shape
    got = gpu.word_rects(pack_bits(m), w, h, *params)[0]
    want = ref.word_rects(pack_bits(m), w, h, *params)
    np.testing.assert_array_equal(got, want)


def test_word_rects_pages_and_device_masks(gpu):
    """Pages in one call equal pages one by one; a device mask equals the host mask; bits past
    the page's width are ignored."""
    import torch

    rng = np.random.default_rng(2)
    h, w = 70, 131
    pages = []
    for i in range(4):
        m = np.zeros((h, w), bool)
        for _ in range(12 * i):
            y, x = rng.integers(0, h - 6), rng.integers(0, w - 20)
            m[y:y + rng.integers(2, 7), x:x + rng.integers(3, 20)] = True
        pages.append(pack_bits(m))
    bits = np.stack(pages)
    bits[..., -1] |= np.uint32(0xffffffff << (w % 32) & 0xffffffff)  # set bits past the width are ignored
    got = gpu.word_rects(bits, w, h)
    assert len(got) == 4 and len(got[0]) == 0
    d = torch.from_numpy(bits.view(np.int32)).cuda()
    dev = gpu.word_rects(None, w, h, d_mask=d.data_ptr(), n=4)
    for g, dv, b in zip(got, dev, pages):
        want = ref.word_rects(b, w, h)
        np.testing.assert_array_equal(g, want)
        np.testing.assert_array_equal(dv, want)


def _comb_disk(r=1100, size=2500, seed=4):
    """A disk with a ragged rim (radius jittered by +-8 px every 0.1 degrees): thousands of
    Douglas-Peucker points outside the octagon of extremes, past the shared-memory sort."""
    rng = np.random.default_rng(seed)
    jit = rng.integers(-8, 9, 3600)
    yy, xx = np.mgrid[:size, :size]
    ang = (np.degrees(np.arctan2(yy - size / 2, xx - size / 2)) % 360 / 0.1).astype(int) % 3600
    return np.hypot(yy - size / 2, xx - size / 2) <= r + jit[ang]


def test_word_rects_large_components(gpu):
    """One large component with a ragged rim (the global-memory sort), and a page of word blobs
    (the benchmark's masks)."""
    for m in (_comb_disk(), synth.page_word_mask(2003)):
        h, w = m.shape
        bits = pack_bits(m)
        np.testing.assert_array_equal(gpu.word_rects(bits, w, h)[0], ref.word_rects(bits, w, h))


def test_word_rects_detection_mask(gpu):
    """A config 1 page through the detector, then its mask's word rectangles."""
    det = wocr.Detector(gpu, synth.ocrs_det_model())
    try:
        page = synth.page(5, 2550, 3300)
        bits = det.detect_page(page, 2550, 3300, 0.5)
    finally:
        det.close()
    got = gpu.word_rects(bits, 2550, 3300)[0]
    want = ref.word_rects(bits, 2550, 3300)
    assert len(want) > 0
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("seed,thresh", [(1, 0.3), (2, 0.2), (3, 0.5)])
def test_db_boxes_bit_exact(gpu, seed, thresh):
    """ppdet::boxes on the device (`wocr_db_boxes`, host and device maps) equals the C
    restatement: the same boxes, bit for bit, in the same reading order."""
    import torch

    from _helpers import db_map

    prob = db_map(seed)
    tp = (3.4647, 3.4375)
    want = ref.db_boxes(prob, tp, thresh)
    assert len(want) > 10
    np.testing.assert_array_equal(gpu.db_boxes(prob, tp, thresh), want)
    d = torch.from_numpy(prob).cuda()
    np.testing.assert_array_equal(gpu.db_boxes(None, tp, thresh, d_prob=d.data_ptr(), w=prob.shape[1],
                                               h=prob.shape[0]), want)


def test_ppdet_boxes_on_detector_map(gpu):
    """The DB boxes of a config 4 page's map, straight from the detector's resident map."""
    g = wocr.NdGraph(gpu, synth.pp_det_model())
    try:
        prob, tp = g.ppdet_page(synth.page(3, 1275, 1650), 1275, 1650, 960)
        got = g.db_boxes(0.3)
    finally:
        g.close()
    np.testing.assert_array_equal(got, ref.db_boxes(prob, tp, 0.3))


def _check_pipeline(gpu, det, page, w, h, min_lines, min_batches):
    """wocr_pp_page against its stages: its boxes are the DB boxes of the detector's map
    (bit-exact), and each line's arg-max classes equal the oracle's recognition of the same line
    images (up to near-ties at the oracle's precision), line by line in reading order."""
    from _helpers import argmax_parity, max_ties

    rec = synth.pp_rec_model()
    with wocr.PPPipeline(gpu, det, rec) as pp:
        boxes, bests = pp.page(page, w, h)
    g = wocr.NdGraph(gpu, det)
    try:
        prob, tp = g.ppdet_page(page, w, h, 960)
    finally:
        g.close()
    np.testing.assert_array_equal(boxes, ref.db_boxes(prob, tp, 0.3))
    assert len(bests) == len(boxes) >= min_lines
    batches, order = ref.pp_batches(page, ref.pp_line_rects(boxes, 0.1))
    assert len(batches) >= min_batches
    k = steps = ties_all = 0
    for data, n, width in batches:
        logits = ref.run_onnx(rec, data, stop_before_softmax=True)
        T = logits.shape[1]
        for j in range(n):
            line = order[k + j]
            assert len(bests[line]) == T
            bad, ties = argmax_parity(bests[line], logits[j])
            assert bad == 0, f"line {line}: {bad} steps differ"
            steps += T
            ties_all += ties
        k += n
    assert ties_all <= max_ties(steps), f"{ties_all} near-tie steps of {steps}"


def test_pp_page_pipeline(gpu):
    """The PP-OCRv6 page pipeline with the random-init DB detector (one page-sized box)."""
    _check_pipeline(gpu, synth.pp_det_model(), synth.page(6, 1275, 1650), 1275, 1650, 1, 1)


def test_pp_page_pipeline_many_lines(gpu):
    """The pipeline with a detector that marks word blobs: over a hundred boxes in reading order,
    recognised in width-sorted batches whose results must come back to the right lines."""
    _check_pipeline(gpu, synth.pp_ink_det_model(), synth.page(6, 1275, 1650, bands=10), 1275, 1650, 100, 5)


def test_pp_page_pipeline_full_size(gpu):
    """Config 4's page size (2550 x 3300): the random-init DB detector (one page-sized box, a
    two-pass cut of a tall crop) and the ink detector (hundreds of boxes, dozens of batches)."""
    _check_pipeline(gpu, synth.pp_det_model(), synth.page(3000, 2550, 3300), 2550, 3300, 1, 1)
    _check_pipeline(gpu, synth.pp_ink_det_model(), synth.page(3001, 2550, 3300), 2550, 3300, 500, 30)


def test_db_boxes_at_the_score_threshold(gpu):
    """box_thresh equal to boxes' exact scores (and one ulp either side): the order-free bound
    cannot settle those boxes, so the ordered score decides, and the boxes still equal the
    oracle's."""
    from _helpers import db_map

    prob = db_map(4)
    h, w = prob.shape
    tp = (3.4647, 3.4375)
    rects = ref.word_rects(pack_bits(prob > np.float32(0.3)), w, h, 0.0, 0.0, -np.inf)
    rects = rects[np.minimum(rects[:, 4], rects[:, 5]) >= 3]
    scores = ref.db_scores(prob, rects)
    for s in scores[:: max(1, len(scores) // 6)]:
        for t in (np.nextafter(s, np.float32(-1)), s, np.nextafter(s, np.float32(2))):
            want = ref.db_boxes(prob, tp, 0.3, float(t))
            np.testing.assert_array_equal(gpu.db_boxes(prob, tp, 0.3, float(t)), want)


def test_post_processing_argument_errors(gpu):
    """The C entry points of the post-processing reject what they cannot do with a status and a
    message, as the reference returns Err: a short output buffer (counts still filled, so the
    caller can size it), pages past 32,767 pixels, a map that is neither given nor computed,
    missing outputs."""
    import ctypes

    lib = wocr.lib()
    m = word_masks()[2]
    h, w = m.shape
    bits = pack_bits(m)
    want = ref.word_rects(bits, w, h)
    counts = np.zeros(1, np.int32)
    out = np.zeros((1, 6), np.float32)
    st = lib.wocr_word_rects(gpu.h, bits.ctypes.data, 1, w, h, 0, 3.0, 0.0, 100.0, out.ctypes.data, 1,
                             counts.ctypes.data)
    assert st == 8 and counts[0] == len(want) > 1 and b"rects holds 1" in lib.wocr_last_error()
    st = lib.wocr_word_rects(gpu.h, bits.ctypes.data, 1, 40000, h, 0, 3.0, 0.0, 100.0, None, 0, counts.ctypes.data)
    assert st == 1 and b"32767" in lib.wocr_last_error()
    st = lib.wocr_word_rects(gpu.h, bits.ctypes.data, 1, w, h, 0, 3.0, 0.0, 100.0, None, 0, None)
    assert st == 1

    prob = np.random.default_rng(0).random((40, 30), dtype=np.float32)
    tp = np.float32([1, 1])
    n = ctypes.c_int32()
    st = lib.wocr_db_boxes(gpu.h, prob.ctypes.data, 30, 40, 0, tp.ctypes.data, 0.2, 0.45, 1.4, 3.0, None, 0,
                           ctypes.byref(n))
    assert st == 0
    if n.value > 0:
        st = lib.wocr_db_boxes(gpu.h, prob.ctypes.data, 30, 40, 0, tp.ctypes.data, 0.2, 0.45, 1.4, 3.0,
                               out.ctypes.data, 0, ctypes.byref(n))
        assert st == 8
    st = lib.wocr_db_boxes(gpu.h, prob.ctypes.data, 0, 40, 0, tp.ctypes.data, 0.2, 0.45, 1.4, 3.0, None, 0,
                           ctypes.byref(n))
    assert st == 1 and b"map size" in lib.wocr_last_error()

    g = wocr.NdGraph(gpu, synth.pp_det_model())
    try:
        st = lib.wocr_ppdet_boxes(g.h, 0.2, 0.45, 1.4, 3.0, None, 0, ctypes.byref(n))
        assert st == 1 and b"wocr_ppdet_page first" in lib.wocr_last_error()
    finally:
        g.close()
    with wocr.PPPipeline(gpu, synth.pp_det_model(), synth.pp_rec_model()) as pp:
        db = np.float32([0.3, 0.45, 1.4, 3.0])
        page = synth.page(1, 200, 300)
        st = lib.wocr_pp_page(pp.h, page.ctypes.data, 200, 300, 960, db.ctypes.data, 0.1, 0, None, 0,
                              ctypes.byref(n), None, 0, None)
        assert st == 1 and b"batch" in lib.wocr_last_error()
        st = lib.wocr_pp_page(pp.h, page.ctypes.data, 200, 300, 960, db.ctypes.data, 0.1, 16, None, 0,
                              ctypes.byref(n), None, 0, None)
        assert st == 0 and n.value >= 0                       # boxes only: best = NULL, cap = 0
