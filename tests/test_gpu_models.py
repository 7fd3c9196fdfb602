"""Whole-model parity of the CUDA path against the CPU oracle on the benchmark configurations'
seeded synthetic models and inputs (tolerances in tests/_helpers.py)."""
import numpy as np
import pytest

import wocr
from oracle import ref
from wocr import synth

from _helpers import PROB_TOL, argmax_parity, gru_r16, mask_parity, max_ties, softmax

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def det_model():
    return synth.ocrs_det_model()


@pytest.fixture(scope="module")
def detector(gpu, det_model):
    d = wocr.Detector(gpu, det_model)
    yield d
    d.close()


@pytest.mark.parametrize("w,h", [(2550, 3300), (517, 389), (600, 1700)])
def test_detect_page(detector, det_model, w, h):
    """Config 1 (ocrs detection), and pages smaller than the model (padding path, width not a
    multiple of 32)."""
    page = synth.page(11, w, h)
    thr = 0.5
    bits = detector.detect_page(page, w, h, thr)
    rbits, prob, _ = ref.detect_page(det_model, page, thr)
    bad, band = mask_parity(bits, rbits, prob, thr, w)
    assert bad == 0, f"{bad} mask pixels differ outside the threshold band ({band} in it)"


@pytest.mark.parametrize("w,h", [(1275, 1650), (640, 1999)])
def test_detect_pages_compacted_upload(detector, det_model, w, h):
    """Tall pages go up compacted to the rows the grey/resize reads (1650 rows: period 16 output
    rows / 33 page rows); a height with no short period (1999) goes up whole.  Masks match the
    oracle and the single-page path, and the reported upload bytes say which path ran."""
    pages = np.stack([synth.page(40 + k, w, h) for k in range(2)])
    many = detector.detect_pages(pages, 0.5)
    h2d, d2h = detector.last_transfer_bytes()
    assert d2h == many.nbytes
    if h == 1650:
        assert h2d == 2 * 800 * 2 * w * 3  # two pages, 1600 rows each
    else:
        assert h2d == pages.nbytes
    for k in range(2):
        rbits, prob, _ = ref.detect_page(det_model, pages[k], 0.5)
        bad, band = mask_parity(many[k], rbits, prob, 0.5, w)
        assert bad == 0, f"page {k}: {bad} mask pixels differ outside the threshold band ({band} in it)"


def test_detect_pages_batched_equals_single(detector):
    pages = np.stack([synth.page(20 + k, 640, 480) for k in range(3)])
    many = detector.detect_pages(pages, 0.5)
    for k in range(3):
        one = detector.detect_page(pages[k], 640, 480, 0.5)
        assert (many[k] == one).all()


def test_detect_pages_graph_replay(detector, monkeypatch):
    """Repeated calls replay captured CUDA graphs (the upload chunks and a last, shorter one);
    the masks equal those of direct launches, and changing the input between replays is seen."""
    pages = np.stack([synth.page(30 + k, 700, 560) for k in range(7)])
    first = detector.detect_pages(pages, 0.5)
    again = detector.detect_pages(pages, 0.5)
    assert (first == again).all()
    other = np.ascontiguousarray(pages[::-1])
    swapped = detector.detect_pages(other, 0.5)
    assert (swapped == first[::-1]).all()
    monkeypatch.setenv("WOCR_NO_GRAPH", "1")
    direct = detector.detect_pages(pages, 0.5)
    assert (direct == first).all()
    monkeypatch.setenv("WOCR_DETECT_CHUNK", "0")
    whole = detector.detect_pages(pages, 0.5)
    assert (whole == first).all()


def test_detect_prob_map(detector, det_model):
    x = ref.grey_resize(synth.page(5, 1275, 1650)).reshape(1, 1, 800, 600)
    got = detector.detect(x)
    want = ref.detect(det_model, x)[0, 0]
    assert np.abs(got - want).max() < 1e-4


@pytest.fixture(scope="module")
def rec_model():
    return synth.ocrs_rec_model()


@pytest.mark.parametrize("n", [1, 9, 64])
def test_recognize(gpu, rec_model, n):
    """Config 0 (ocrs recognition): per-line lengths, lines batched as ocr-bench batches them.  The
    recurrent weights are fp16 as on the reference's GPU path, so the arg-max is checked against
    the oracle with the same fp16 R and against the fp32 oracle (rten): every step's class is the
    oracle's or a near-tie, the near-ties are at most max_ties (measured on the 64 seeded lines:
    none against the fp32 oracle, one step of 8,409 against the fp16 one, a step on which the two
    oracles disagree themselves), the probabilities are within PROB_TOL of the fp32 oracle's and
    the greedy CTC text is the fp32 oracle's."""
    lines = synth.ocrs_lines(0, n=n)
    batches, order, widths = synth.ocrs_batches(lines)
    rec = wocr.Recognizer(gpu, rec_model)
    try:
        logits, tmax, lens, best = rec.recognize(batches)
    finally:
        rec.close()
    rlogits, rtmax, rlens = ref.recognize(rec_model, batches)
    hlogits, _, _ = ref.recognize(gru_r16(rec_model), batches)
    assert tmax == rtmax and lens == rlens
    steps = ties16 = ties32 = 0
    for line in range(len(lens)):
        t = lens[line]
        g, r = logits[:t, line], rlogits[:t, line]
        bad, ties = argmax_parity(best[:t, line], hlogits[:t, line])
        assert bad == 0, f"line {line}: {bad} steps choose another class"
        ties16 += ties
        bad, ties = argmax_parity(best[:t, line], r)
        assert bad == 0, f"line {line}: {bad} steps choose another class than the fp32 oracle"
        ties32 += ties
        steps += t
        assert np.abs(softmax(g) - softmax(r)).max() < PROB_TOL
    assert ties16 <= max_ties(steps), f"{ties16} near-tie steps of {steps} against the fp16-R oracle"
    assert ties32 <= max_ties(steps), f"{ties32} near-tie steps of {steps} against the fp32 oracle"
    # greedy CTC text identical
    for k, line in enumerate(range(len(lens))):
        want = ref.ocrs_decode(rlogits, line, lens[line], widths[k], synth.OCRS_ALPHABET)
        got = wocr.ocrs_decode(best[:, line], lens[line], widths[k], synth.OCRS_ALPHABET)
        assert got == want


@pytest.fixture(scope="module")
def pp_model():
    return synth.pp_rec_model()


def test_pp_recognition(gpu, pp_model):
    """Config 3 (PP-OCRv6-style recognition, 18,709 classes), all 256 lines in their 16 width
    batches: the arg-max identical to the oracle's at every step (no near-tie excused) and the
    chosen class's probability within PROB_TOL."""
    lines = synth.pp_lines(2, n=256)
    batches, order = synth.pp_batches(lines)
    assert len(batches) == 16
    g = wocr.NdGraph(gpu, pp_model, stop_before_softmax=True)
    steps = ties_all = 0
    try:
        for data, n, w in batches:
            best, mx, lse, shape = g.argmax(data)
            logits = ref.run_onnx(pp_model, data, stop_before_softmax=True)
            assert shape == logits.shape
            flat = logits.reshape(-1, logits.shape[-1])
            bad, ties = argmax_parity(best, flat)
            assert bad == 0, f"{bad} of {len(best)} steps choose another class ({ties} near-ties)"
            steps += len(best)
            ties_all += ties
            rb, t1, _, rlse = ref.argmax(flat)
            p_gpu = np.exp(mx - lse)
            p_ref = np.exp(t1 - rlse)
            assert np.abs(p_gpu - p_ref).max() < PROB_TOL
    finally:
        g.close()
    assert steps > 20000
    assert ties_all == 0, f"{ties_all} of {steps} steps choose another class (near-ties)"


def test_pp_detection(gpu):
    """Config 4 (PP-OCRv6-style DB detection): det_input on the device and the probability map."""
    m = synth.pp_det_model()
    page = synth.page(3, 2550, 3300)
    x, tp = wocr.NdGraph.det_input(gpu, page, 2550, 3300, 960)
    rx, rtp = ref.det_input(page, 960)
    assert x.shape == rx.shape == (1, 3, 960, 736)
    assert np.abs(x - rx).max() < 1e-5
    assert np.allclose(tp, rtp)
    g = wocr.NdGraph(gpu, m)
    try:
        prob, tp2 = g.ppdet_page(page, 2550, 3300, 960)
    finally:
        g.close()
    want = ref.run_onnx(m, rx)[0, 0]
    assert prob.shape == want.shape
    assert np.abs(prob - want).max() < 1e-4


def _db_rects(rng, w, h, n):
    """Rotated boxes [cx, cy, up_x, up_y, width, height] over a w x h map: random ones, boxes on
    and past every edge, an empty one, a tiny one, a NaN one and one larger than the map."""
    ang = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    r = np.stack([rng.uniform(0, w, n), rng.uniform(0, h, n), np.sin(ang), -np.cos(ang),
                  rng.uniform(2, 200, n), rng.uniform(2, 40, n)], 1).astype(np.float32)
    edge = [[0, 0, 0, -1, 30, 12], [w - 1, h - 1, 0, -1, 40, 9], [w + 30, h / 2, 0, -1, 20, 20],
            [w / 2, -5, 0.6, -0.8, 50, 15], [w / 2, h / 2, 0, -1, 0, 0], [7.3, 9.6, 0.7071, -0.7071, 1, 1],
            [float("nan"), 4, 0, -1, 5, 5], [w / 2, h / 2, 0, -1, 1e7, 1e7]]
    return np.concatenate([r, np.float32(edge)])


def test_pp_db_mask_and_scores(gpu):
    """DB post-processing on the device-resident map (src/ppdet.rs:63-92): the threshold bit mask
    equals `prob > thresh` and every box score equals the CPU restatement to the bit, after the
    first call and after a graph replay with another page."""
    m = synth.pp_det_model()
    rng = np.random.default_rng(11)
    g = wocr.NdGraph(gpu, m)
    try:
        for seed in (3, 4):
            page = synth.page(seed, 1275, 1650)
            prob, _ = g.ppdet_page(page, 1275, 1650, 960)
            h, w = prob.shape
            for thr in (0.2, float(np.median(prob))):
                bits = g.db_mask(thr)
                assert bits.shape == (h, (w + 31) // 32)
                on = np.zeros((h, bits.shape[1] * 32), bool)
                on[:, :w] = prob > np.float32(thr)
                want = np.packbits(on.reshape(h, -1, 32), axis=2, bitorder="little").view("<u4")[..., 0]
                np.testing.assert_array_equal(bits, want)
            rects = _db_rects(rng, w, h, 300)
            got = g.db_scores(rects)
            np.testing.assert_array_equal(got, ref.db_scores(prob, rects))
            assert len(g.db_scores(np.zeros((0, 6), np.float32))) == 0
    finally:
        g.close()


def test_ndgraph_replay(gpu, pp_model, monkeypatch):
    """NdGraph calls of a known shape replay a captured CUDA graph (run, arg-max and the PP
    detection page): the results equal direct runs, and new input values are seen."""
    from wocr.synth import _Builder, _svtr_block
    b = _Builder(21)
    y = b.linear(b.layer_norm(_svtr_block(b, "x"), 120), 120, 37)
    m = b.model("x", y)
    rng = np.random.default_rng(5)
    x1 = rng.standard_normal((2, 9, 120)).astype(np.float32)
    x2 = rng.standard_normal((2, 9, 120)).astype(np.float32)
    g = wocr.NdGraph(gpu, m)
    try:
        outs = [g.run(x) for x in (x1, x1, x2, x1)]          # direct, capture, replay, replay
    finally:
        g.close()
    assert (outs[0] == outs[1]).all() and (outs[0] == outs[3]).all()
    assert np.abs(outs[2] - ref.run_onnx(m, x2)).max() < 2e-4 * max(1.0, float(np.abs(outs[2]).max()))

    data = synth.pp_batches(synth.pp_lines(2, n=16))[0][0][0]
    g = wocr.NdGraph(gpu, pp_model, stop_before_softmax=True)
    try:
        r1, r2, r3 = (g.argmax(data) for _ in range(3))
    finally:
        g.close()
    for a, b2 in ((r1, r2), (r1, r3)):
        assert all((u == v).all() for u, v in zip(a[:3], b2[:3])) and a[3] == b2[3]

    det = synth.pp_det_model()
    page = synth.page(4, 1275, 1650)
    g = wocr.NdGraph(gpu, det)
    try:
        p1, _ = g.ppdet_page(page, 1275, 1650, 960)
        p2, _ = g.ppdet_page(page, 1275, 1650, 960)
        other = synth.page(9, 1275, 1650)
        p3, _ = g.ppdet_page(other, 1275, 1650, 960)
        monkeypatch.setenv("WOCR_NO_GRAPH", "1")
        p4, _ = g.ppdet_page(other, 1275, 1650, 960)
    finally:
        g.close()
    assert (p1 == p2).all() and (p3 == p4).all()


def test_recognize_replay(gpu, rec_model, monkeypatch):
    """wocr_recognize calls of a known batch layout replay a captured CUDA graph: logits and
    arg-max equal those of direct runs, with and without logits, and new line images are seen."""
    batches, _, _ = synth.ocrs_batches(synth.ocrs_lines(3, n=9))
    other = [(np.ascontiguousarray(d[::-1]), n, w) for d, n, w in batches]
    rec = wocr.Recognizer(gpu, rec_model)
    try:
        a = rec.recognize(batches)                       # direct
        b = rec.recognize(batches)                       # capture + replay
        c = rec.recognize(batches)                       # replay
        o = rec.recognize(other)                         # replay on new data
        nb = rec.recognize(batches, want_logits=False)   # another layout (no logits)
        nb2 = rec.recognize(batches, want_logits=False)
        monkeypatch.setenv("WOCR_NO_GRAPH", "1")
        od = rec.recognize(other)
    finally:
        rec.close()
    for x in (b, c):
        assert x[1] == a[1] and x[2] == a[2]
        assert (x[0] == a[0]).all() and (x[3] == a[3]).all()
    assert (o[0] == od[0]).all() and (o[3] == od[3]).all()
    assert (nb[3] == a[3]).all() and (nb2[3] == a[3]).all()


def test_recognizer_rejects_unsupported_models(gpu, rec_model):
    """Recognizer::new's checks (src/gpu.rs:1452-1506): hidden size 256, linear_before_reset = 1,
    bidirectional, exactly two GRU layers, an AveragePool after the trunk; anything else is an
    error with a message, as the reference returns Err."""
    import copy

    grus = [i for i, n in enumerate(rec_model.nodes) if n.op == "GRU"]
    assert len(grus) == 2
    for attr, value in (("hidden_size", 128), ("linear_before_reset", 0), ("direction", "forward")):
        m = copy.deepcopy(rec_model)
        m.nodes[grus[0]].attrs[attr] = value
        with pytest.raises(wocr.WocrError, match="unsupported GRU attributes"):
            wocr.Recognizer(gpu, m)
    m = copy.deepcopy(rec_model)
    del m.nodes[grus[1]]
    with pytest.raises(wocr.WocrError, match="1 GRU layers"):
        wocr.Recognizer(gpu, m)
    m = copy.deepcopy(rec_model)
    for n in m.nodes:
        if n.op == "AveragePool":
            n.op = "MaxPool"
    # the trunk is built up to the AveragePool; without one it runs into the GRU's ops, which
    # the 4-D graph rejects like the reference's Graph::build
    with pytest.raises(wocr.WocrError, match="no AveragePool|unsupported op"):
        wocr.Recognizer(gpu, m)
