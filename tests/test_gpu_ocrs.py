"""The ocrs page pipeline on the device (config 2; src/bin/ocr-bench.rs:458-585 without DET /
REC): line images bit-exact against the oracle's restatement of ocrs' prepare_recognition_input
and line_batches, and whole pages stage by stage against the oracle (the lines found from the
detector's mask, each line's recognition arg-max)."""
import numpy as np
import pytest

import wocr
from _helpers import argmax_parity, gru_r16, max_ties
from oracle import ref
from wocr import synth

pytestmark = pytest.mark.gpu

W, H = 1275, 1650


@pytest.fixture(scope="module")
def rec_model():
    return synth.ocrs_rec_model()


def _small_page(seed):
    return synth.page(seed, W, H, bands=14, line_h=36)


def _lines_of(page, det):
    """The oracle's lines from the mask of the GPU detector (so that the stages after detection are
    compared on the same mask)."""
    gpu = det.gpu
    bits = det.detect_page(page, page.shape[1], page.shape[0], 0.5)
    return ref.ocrs_page_lines(bits, page.shape[1], page.shape[0])


def _check_batches(gpu, page, lines):
    import torch

    d = torch.from_numpy(page).cuda()
    slots, widths, layout, total = gpu.ocrs_lines(d.data_ptr(), page.shape[1], page.shape[0], lines)
    out = torch.empty(max(total, 1), dtype=torch.float32, device="cuda")
    gpu.ocrs_lines(d.data_ptr(), page.shape[1], page.shape[0], lines, d_out=out.data_ptr(), cap=total)
    got = out.cpu().numpy()
    want, order, wwidths = ref.ocrs_line_batches(page, lines)
    assert slots == order and widths == wwidths
    assert layout == [(n, w) for _, n, w in want]
    o = 0
    for data, n, w in want:
        np.testing.assert_array_equal(got[o:o + data.size].reshape(data.shape), data)
        o += data.size
    assert o == total


def test_ocrs_lines_bit_exact_on_detected_lines(gpu):
    det = wocr.Detector(gpu, synth.ocrs_ink_det_model())
    try:
        page = _small_page(21)
        lines = _lines_of(page, det)
    finally:
        det.close()
    assert len(lines) >= 12
    _check_batches(gpu, page, lines)


def test_ocrs_lines_edge_cases(gpu):
    """Rotated and upside-down words, a word whose up axis is horizontal, lines running off every
    page edge, a one-word line narrower than the 10-column minimum and one wider than 800."""
    page = _small_page(22)
    rng = np.random.default_rng(5)
    lines = []
    for k in range(30):
        n = int(rng.integers(1, 7))
        x = float(rng.uniform(-60, W - 100))
        y = float(rng.uniform(-20, H + 10))
        a = float(rng.uniform(-0.25, 0.25))
        ws = []
        for q in range(n):
            w, h = float(rng.uniform(10, 90)), float(rng.uniform(14, 50))
            up = [np.sin(a), -np.cos(a)]
            if q % 3 == 1:
                up = [-up[0], -up[1]]                            # up pointing down
            rect = [x + w / 2, y, up[0], up[1], w, h]
            if q % 5 == 4:                                       # up axis nearer horizontal
                rect = [x + w / 2, y, -np.cos(a), -np.sin(a), h, w]
            ws.append(rect)
            x += w + float(rng.uniform(2, 30))
        lines.append(ref.pad_line(np.array(ws, np.float32)))
    lines.append(np.array([[600, 800, 0, -1, 4, 60]], np.float32))           # W below 10
    lines.append(np.array([[640, 300, 0, -1, 1250, 20]], np.float32))        # W above 800
    _check_batches(gpu, page, lines)


def _oracle_check(gpu, det_model, rec_model, pages, got, min_lines):
    """Each page's lines (padded words) equal the oracle's from the GPU mask, and each line's
    arg-max equals the oracle's recognition of the oracle's own batches, step by step."""
    det = wocr.Detector(gpu, det_model)
    try:
        total_lines = steps = ties_all = 0
        for page, lines in zip(pages, got):
            want = _lines_of(page, det)
            assert len(lines) == len(want)
            for (words, width, best), wl in zip(lines, want):
                np.testing.assert_array_equal(words, wl)
            batches, order, widths = ref.ocrs_line_batches(page, want)
            rl, rt, rlens = ref.recognize(gru_r16(rec_model), batches)   # fp16 R, as the GPU path
            for k, line in enumerate(order):
                words, width, best = lines[line]
                assert width == widths[k]
                assert len(best) == rlens[k]
                bad, ties = argmax_parity(best, rl[:rlens[k], k])
                assert bad == 0, f"line {line}: {bad} steps differ"
                steps += rlens[k]
                ties_all += ties
            total_lines += len(lines)
        assert total_lines >= min_lines
        assert ties_all <= max_ties(steps), f"{ties_all} near-tie steps of {steps}"
    finally:
        det.close()


def test_ocrs_pipeline_against_oracle(gpu, rec_model):
    pages = [_small_page(30 + k) for k in range(3)]
    det_m = synth.ocrs_ink_det_model()
    with wocr.OcrsPipeline(gpu, det_m, rec_model) as p:
        got = p.pages(pages, W, H, merge=2)
    _oracle_check(gpu, det_m, rec_model, pages, got, 30)


def test_ocrs_pipeline_full_size(gpu, rec_model):
    """Config 2's page size (2550 x 3300, 36 text bands) with the ink detector, and the
    config's own random-init detector (seed 1)."""
    pages = [synth.page(1000 + k, 2550, 3300) for k in range(2)]
    for det_m, min_lines in ((synth.ocrs_ink_det_model(), 60), (synth.ocrs_det_model(), 1)):
        with wocr.OcrsPipeline(gpu, det_m, rec_model) as p:
            got = p.pages(pages, 2550, 3300, merge=2)
        _oracle_check(gpu, det_m, rec_model, pages, got, min_lines)


@pytest.mark.parametrize("merge,lanes", [(3, 1), (1, 2), (2, 3)])
def test_ocrs_pages_merge_and_lanes_equal(gpu, rec_model, merge, lanes):
    """Merging recognitions and spreading pages over lanes change nothing in the results, from
    host or from device pages."""
    import torch

    pages = [_small_page(40 + k) for k in range(5)]
    det_m = synth.ocrs_ink_det_model()
    with wocr.OcrsPipeline(gpu, det_m, rec_model) as p:
        want = p.pages(pages, W, H)
        got = p.pages(pages, W, H, merge=merge, lanes=lanes)
        assert p.last_bytes[0] == 5 * W * H * 3
        d = [torch.from_numpy(pg).cuda() for pg in pages]
        torch.cuda.synchronize()
        dev = p.pages([t.data_ptr() for t in d], W, H, merge=merge, lanes=lanes)
        assert p.last_bytes[0] == 0
    for res in (got, dev):
        for a, b in zip(res, want):
            assert len(a) == len(b)
            for (wa, xa, ba), (wb, xb, bb) in zip(a, b):
                np.testing.assert_array_equal(wa, wb)
                assert xa == xb
                np.testing.assert_array_equal(ba, bb)
