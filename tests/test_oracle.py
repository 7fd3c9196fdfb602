"""The CPU oracle against an independent implementation (PyTorch CPU), and its restatement of
the reference's coordinate formulas, on small seeded cases.  No GPU needed."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import ref
from wocr import synth

from _helpers import pack_bits, word_masks

RNG = np.random.default_rng(1234)


def rnd(*shape):
    return RNG.standard_normal(shape).astype(np.float32)


@pytest.mark.parametrize("cin,cout,k,stride,pads,group", [
    (3, 5, 3, (1, 1), (1, 1, 1, 1), 1),
    (4, 6, 3, (2, 2), (1, 1, 1, 1), 1),
    (8, 8, 3, (2, 1), (1, 1, 1, 1), 8),     # depthwise, stride (2, 1)
    (1, 4, 5, (1, 1), (2, 2, 2, 2), 1),
    (6, 3, 1, (1, 1), (0, 0, 0, 0), 1),
    (4, 4, 3, (2, 2), (0, 0, 1, 1), 1),     # asymmetric (SAME_UPPER-like) padding
])
def test_conv2d_vs_torch(cin, cout, k, stride, pads, group):
    x = rnd(2, cin, 11, 13)
    w = rnd(cout, cin // group, k, k)
    b = rnd(cout)
    y = ref.conv2d(x, w, b, group=group, strides=stride, pads=pads)
    xp = F.pad(torch.from_numpy(x), (pads[1], pads[3], pads[0], pads[2]))
    yt = F.conv2d(xp, torch.from_numpy(w), torch.from_numpy(b), stride=stride, groups=group).numpy()
    assert y.shape == yt.shape
    assert np.abs(y - yt).max() < 1e-4


def test_conv2d_epilogue_residual_scale():
    x, w, b = rnd(2, 4, 7, 9), rnd(5, 4, 3, 3), rnd(5)
    res, sc = rnd(2, 5, 7, 9), rnd(2, 4)
    y = ref.conv2d(x, w, b, pads=(1, 1, 1, 1), act=1, res=res, insc=sc)
    xs = torch.from_numpy(x) * torch.from_numpy(sc)[:, :, None, None]
    yt = torch.relu(F.conv2d(xs, torch.from_numpy(w), torch.from_numpy(b), padding=1)) + torch.from_numpy(res)
    assert np.abs(y - yt.numpy()).max() < 1e-4


@pytest.mark.parametrize("act", [0, 1, 2, 3, 4])
def test_activations(act):
    v = np.linspace(-6, 6, 97).astype(np.float32)
    got = np.array([ref.lib().oracle_act(float(x), act) for x in v], np.float32)
    t = torch.from_numpy(v)
    want = {0: t, 1: torch.relu(t), 2: torch.sigmoid(t), 3: F.gelu(t), 4: F.silu(t)}[act].numpy()
    assert np.abs(got - want).max() < 2e-6


def test_erf_as_bound():
    v = np.linspace(-4, 4, 801)
    got = np.array([ref.lib().oracle_erf(float(x)) for x in v])
    want = np.array([math.erf(x) for x in v])
    assert np.abs(got - want).max() < 5e-7   # A&S 7.1.26: 1.5e-7 plus float rounding


def test_convt_vs_torch():
    x, w, b = rnd(2, 6, 5, 7), rnd(6, 4, 2, 2), rnd(4)
    y = ref.convt(x, w, b, stride=2, act=1)
    yt = torch.relu(F.conv_transpose2d(torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b), stride=2))
    assert np.abs(y - yt.numpy()).max() < 1e-4
    w3 = rnd(6, 4, 3, 3)
    y3 = ref.convt(x, w3, None, stride=2)
    yt3 = F.conv_transpose2d(torch.from_numpy(x), torch.from_numpy(w3), stride=2)
    assert np.abs(y3 - yt3.numpy()).max() < 1e-4


def test_pool_vs_torch():
    x = rnd(2, 3, 9, 12)
    y = ref.pool(x, 2, 2, 2, 2)
    assert np.abs(y - F.max_pool2d(torch.from_numpy(x), 2).numpy()).max() == 0
    y = ref.pool(x, 3, 1, 3, 1)
    assert np.abs(y - F.max_pool2d(torch.from_numpy(x), (3, 1)).numpy()).max() == 0
    y = ref.pool(x, 3, 3, 2, 2, pads=(1, 1, 1, 1), avg=True)
    yt = F.avg_pool2d(torch.from_numpy(x), 3, 2, padding=1, count_include_pad=False).numpy()
    assert np.abs(y - yt).max() < 1e-5


def test_gru_vs_torch():
    """ONNX GRU (z, r, h; linear_before_reset = 1) == torch GRU (r, z, n) after a gate reorder."""
    T, n, inp, hid = 7, 3, 16, 256
    X = rnd(T, n, inp) * 0.5
    W = RNG.uniform(-1 / 16, 1 / 16, (2, 3 * hid, inp)).astype(np.float32)
    R = RNG.uniform(-1 / 16, 1 / 16, (2, 3 * hid, hid)).astype(np.float32)
    B = RNG.uniform(-1 / 16, 1 / 16, (2, 6 * hid)).astype(np.float32)
    Y = ref._onnx_gru(X, W, R, B, hid)                       # [T, 2, n, hid]
    g = torch.nn.GRU(inp, hid, bidirectional=True)
    order = lambda a: np.concatenate([a[hid:2 * hid], a[:hid], a[2 * hid:]])  # z,r,h -> r,z,n
    with torch.no_grad():
        for d, sfx in ((0, ""), (1, "_reverse")):
            getattr(g, "weight_ih_l0" + sfx).copy_(torch.from_numpy(order(W[d])))
            getattr(g, "weight_hh_l0" + sfx).copy_(torch.from_numpy(order(R[d])))
            getattr(g, "bias_ih_l0" + sfx).copy_(torch.from_numpy(order(B[d, :3 * hid])))
            getattr(g, "bias_hh_l0" + sfx).copy_(torch.from_numpy(order(B[d, 3 * hid:])))
        yt, _ = g(torch.from_numpy(X))
    yt = yt.numpy().reshape(T, n, 2, hid).transpose(0, 2, 1, 3)
    assert np.abs(Y - yt).max() < 1e-5


def test_gru_lengths():
    """Per-line lengths: steps t >= len are not written, the backward pass starts at len - 1."""
    hid, tmax = 256, 6
    g = rnd(tmax, 2, 2 * 3 * hid) * 0.3
    r = RNG.uniform(-1 / 16, 1 / 16, (2, 3 * hid, hid)).astype(np.float32)
    rb = RNG.uniform(-1 / 16, 1 / 16, (2, 3 * hid)).astype(np.float32)
    y = ref.gru(g, r, rb, [6, 3], hid)
    assert np.isnan(y[3:, 1]).all() and not np.isnan(y[:3, 1]).any() and not np.isnan(y).any(axis=2)[:, 0].any()
    # line 1 alone with tmax 3 gives the same first 3 steps
    y1 = ref.gru(g[:3, 1:2], r, rb, [3], hid)
    assert np.abs(y1[:, 0] - y[:3, 1]).max() == 0


def test_layer_norm_softmax_argmax():
    x = rnd(5, 120)
    g, b = rnd(120), rnd(120)
    y = ref.layer_norm(x, g, b, 1e-6)
    yt = F.layer_norm(torch.from_numpy(x), (120,), torch.from_numpy(g), torch.from_numpy(b), 1e-6).numpy()
    assert np.abs(y - yt).max() < 1e-4
    s = ref.softmax(x)
    assert np.abs(s - torch.softmax(torch.from_numpy(x), -1).numpy()).max() < 1e-6
    xt = x.copy()
    xt[0, 7] = xt[0, 9] = 100.0
    best, t1, t2, lse = ref.argmax(xt)
    assert best[0] == 7 and t1[0] == 100.0 and t2[0] == 100.0          # ties -> lowest index
    assert ref.ocrs_best(xt[0]) == 9                                    # Rust max_by -> last index
    assert np.abs(lse - torch.logsumexp(torch.from_numpy(xt), -1).numpy()).max() < 1e-4


def test_grey_resize_formula():
    """Identity-size resize reproduces the grey formula; out-of-page pixels are -0.5."""
    rgb = RNG.integers(0, 256, (800, 600, 3), dtype=np.uint8)
    g = ref.grey_resize(rgb)
    want = -0.5 + rgb[..., 0] * (0.299 / 255) + rgb[..., 1] * (0.587 / 255) + rgb[..., 2] * (0.114 / 255)
    assert np.abs(g - want).max() < 1e-5
    small = RNG.integers(0, 256, (400, 300, 3), dtype=np.uint8)       # padded to 800 x 600
    g2 = ref.grey_resize(small)
    assert (g2[450:, :] == -0.5).all() and (g2[:, 350:] == -0.5).all()


def test_mask_bits_layout():
    m = np.zeros((800, 600), np.float32)
    m[:, :300] = 1.0
    bits, prob = ref.mask_up(m, 600, 800, 70, 40, 0.5)     # page 70 x 40: 3 words per row
    assert bits.shape == (40, 3)
    for y in range(40):
        row = [(bits[y, x // 32] >> (x % 32)) & 1 for x in range(70)]
        assert row == [int(p > 0.5) for p in prob[y]]
    assert (bits[:, 2] >> 6).max() == 0                     # bits past the page width stay 0


def test_det_input_sizes():
    # the config-4 page: 2550 x 3300 at max_side 960 -> 736 x 960
    assert ref.det_input_size(2550, 3300, 960) == (736, 960)
    assert ref.det_input_size(100, 50, 960) == (96, 64)
    assert ref.det_input_size(10, 10, 960) == (32, 32)


def test_resize_nearest_vs_torch():
    x = rnd(1, 3, 5, 7)
    y = ref.resize_nearest(x, 2.0, 2.0)
    yt = F.interpolate(torch.from_numpy(x), scale_factor=2, mode="nearest").numpy()
    assert np.abs(y - yt).max() == 0


def test_run_onnx_shapes():
    """The interpreter runs every synthetic architecture end to end with the expected shapes."""
    m = synth.ocrs_rec_model()
    lines = synth.ocrs_lines(n=3, wmin=64, wmax=96)
    batches, order, widths = synth.ocrs_batches(lines)
    out = ref.run_onnx(m, batches[0][0])
    assert out.shape == (batches[0][2] // 4, batches[0][1], 97)
    pm = synth.pp_rec_model(classes=50)
    x = np.zeros((2, 3, 48, 64), np.float32)
    y = ref.run_onnx(pm, x)
    assert y.shape == (2, 8, 50) and np.allclose(y.sum(-1), 1.0, atol=1e-5)
    logits = ref.run_onnx(pm, x, stop_before_softmax=True)
    assert np.abs(ref.softmax(logits) - y).max() < 1e-6
    dm = synth.pp_det_model()
    z = ref.run_onnx(dm, np.zeros((1, 3, 64, 96), np.float32))
    assert z.shape == (1, 1, 64, 96)


def test_synth_determinism():
    a, b = synth.page(3, 300, 200), synth.page(3, 300, 200)
    assert (a == b).all()
    la, lb = synth.ocrs_lines(5, n=4), synth.ocrs_lines(5, n=4)
    assert all((x == y).all() for x, y in zip(la, lb))
    ma, mb = synth.ocrs_det_model(), synth.ocrs_det_model()
    assert all((ma.weights[k] == mb.weights[k]).all() for k in ma.weights)


def _tri_resize_np(crop, ow, oh):
    """The image crate's two-pass Triangle resize, restated independently with numpy float32:
    a vertical pass into an f32 image, then a horizontal pass clamped and rounded to u8."""
    def taps(n_in, n_out, o):
        ratio = np.float32(n_in) / np.float32(n_out)
        s = max(ratio, np.float32(1.0))
        c = (np.float32(o) + np.float32(0.5)) * ratio
        left = int(min(max(np.floor(c - s), 0), n_in - 1))
        right = int(min(max(np.ceil(c + s), left + 1), n_in))
        c = c - np.float32(0.5)
        ws = [np.float32(max(np.float32(0), np.float32(1) - abs((np.float32(i) - c) / s))) for i in range(left, right)]
        tot = np.float32(0)
        for wv in ws:
            tot = np.float32(tot + wv)
        return left, [np.float32(wv / tot) for wv in ws]

    ch, cw, _ = crop.shape
    tmp = np.zeros((oh, cw, 3), np.float32)
    for y in range(oh):
        left, ws = taps(ch, oh, y)
        acc = np.zeros((cw, 3), np.float32)
        for i, wv in enumerate(ws):
            acc = (acc + crop[left + i].astype(np.float32) * wv).astype(np.float32)
        tmp[y] = acc
    out = np.zeros((oh, ow, 3), np.uint8)
    for x in range(ow):
        left, ws = taps(cw, ow, x)
        acc = np.zeros((oh, 3), np.float32)
        for j, wv in enumerate(ws):
            acc = (acc + tmp[:, left + j] * wv).astype(np.float32)
        out[:, x] = np.floor(np.clip(acc, 0, 255) + np.float32(0.5)).astype(np.uint8)
    return out


@pytest.mark.parametrize("rect", [[5, 7, 125, 40], [0, 0, 33, 90], [40, 60, 44, 63], [10, 3, 300, 4]])
def test_pp_line_oracle_matches_two_pass_restatement(rect):
    """oracle_pp_line (one output pixel at a time, vertical sums per horizontal tap) equals the
    two-pass resize with an intermediate image, and the line's width and normalisation."""
    rng = np.random.default_rng(5)
    page = rng.integers(0, 256, (120, 320, 3), dtype=np.uint8)
    got = ref.pp_line(page, rect)
    l, t, r, b = (int(min(max(v, 0), lim)) for v, lim in zip(rect, (320, 120, 320, 120)))
    cw, ch = max(r - l, 1), max(b - t, 1)
    ow = int(min(max(np.ceil(np.float32(48) * np.float32(cw) / np.float32(ch)), 8), 3200))
    assert got.shape == (3, 48, ow)
    px = _tri_resize_np(page[t:t + ch, l:l + cw], ow, 48)
    want = ((px.astype(np.float32) / np.float32(255) - np.float32(0.5)) / np.float32(0.5)).transpose(2, 0, 1)
    np.testing.assert_array_equal(got, want)


def _db_score_loops(prob, r):
    """`score` (src/ppdet.rs:63-83) over every pixel of the map, in f32 scalars: the inside test
    alone selects, so the scan rectangle of the oracle must cover every pixel that passes."""
    f = np.float32
    cx, cy, ux, uy, hw, hh = f(r[0]), f(r[1]), f(r[2]), f(r[3]), f(r[4]) / f(2), f(r[5]) / f(2)
    s, n = f(0), 0
    for y in range(prob.shape[0]):
        dy = f(y) - cy
        for x in range(prob.shape[1]):
            dx = f(x) - cx
            if abs(dx * ux + dy * uy) <= hh and abs(dx * -uy + dy * ux) <= hw:
                s = f(s + prob[y, x])
                n += 1
    return f(0) if n == 0 else f(s / f(n))


def test_db_score_oracle_matches_full_scan():
    """oracle_db_score (a scan of the box's bounding rectangle) equals the sum over the whole map,
    for rotated, axis-aligned, clamped, off-map, empty and NaN boxes."""
    rng = np.random.default_rng(3)
    prob = rng.random((37, 53), dtype=np.float32)
    a = np.float32(0.3)
    rects = [[20.5, 14.0, 0, -1, 30, 6], [26.0, 18.0, np.sin(a), -np.cos(a), 25, 9], [1.0, 2.0, 0, -1, 9, 9],
             [52.0, 36.0, -0.6, -0.8, 12, 7], [80.0, 60.0, 0, -1, 10, 10], [10.0, 10.0, 0, -1, 0, 0],
             [10.3, 10.6, 0.70710678, -0.70710678, 1.0, 1.0], [float("nan"), 3.0, 0, -1, 4, 4],
             [26.0, 18.0, 0, -1, 1e9, 1e9]]
    got = ref.db_scores(prob, rects)
    want = np.array([_db_score_loops(prob, r) for r in rects], np.float32)
    np.testing.assert_array_equal(got, want)
    assert got[4] == 0 and got[7] == 0


@pytest.mark.parametrize("k", range(5))
def test_contour_oracle_vs_labelling(k):
    """oracle_contours (Suzuki-Abe border following, External) against scipy's labelling: one
    contour per 8-connected component whose surrounding 4-connected background reaches the
    frame, starting at its first pixel in raster order, made of 8-adjacent steps (closed), and
    visiting exactly the component's pixels that touch (4-neighbour) that background."""
    from scipy import ndimage

    m = word_masks()[k]
    h, w = m.shape
    cs = ref.contours(pack_bits(m), w, h)
    fg, nf = ndimage.label(m, structure=np.ones((3, 3)))
    pad = np.pad(~m, 1, constant_values=True)
    bg, _ = ndimage.label(pad, structure=[[0, 1, 0], [1, 1, 1], [0, 1, 0]])
    frame = bg[0, 0]
    want = []
    for lab in range(1, nf + 1):
        ys, xs = np.nonzero(fg == lab)
        i = np.lexsort((xs, ys))[0]
        y0, x0 = ys[i], xs[i]
        if bg[y0 + 1, x0] == frame:                       # the pixel left of the start (padded coords)
            want.append((y0, x0, lab))
    want.sort()
    assert len(cs) == len(want)
    for c, (y0, x0, lab) in zip(cs, want):
        assert tuple(c[0]) == (x0, y0)
        if len(c) > 1:
            steps = np.abs(np.diff(np.vstack([c, c[:1]]), axis=0))
            assert (steps.max(1) == 1).all()
        comp = fg == lab
        outer = np.zeros_like(comp)
        for dy, dx in ((0, 1), (0, -1), (1, 0), (-1, 0)):
            outer |= np.roll(np.roll(bg == frame, dy, 0), dx, 1)[1:-1, 1:-1]
        border = comp & outer
        got = np.zeros_like(comp)
        got[c[:, 1], c[:, 0]] = True
        assert (got == border).all()


def test_word_rects_oracle_properties():
    """Each rectangle of oracle_word_rects holds its contour's simplified points (so the
    expanded rectangle holds the whole word up to the simplification's 2 px), has a unit up axis,
    and its area passes the filter; a 1 x 1 blob collapses (one point) and is dropped."""
    m = word_masks()[2]
    h, w = m.shape
    r = ref.word_rects(pack_bits(m), w, h)
    assert len(r) > 5
    assert np.allclose(np.hypot(r[:, 2], r[:, 3]), 1, atol=1e-6)
    assert (r[:, 4] * r[:, 5] >= 100).all()
    ys, xs = np.nonzero(m)
    for cx, cy, ux, uy, rw, rh in r:
        along = (xs - cx) * ux + (ys - cy) * uy
        across = (xs - cx) * -uy + (ys - cy) * ux
        inside = (np.abs(along) <= rh / 2 + 1e-3) & (np.abs(across) <= rw / 2 + 1e-3)
        assert inside.sum() >= 3
    one = np.zeros((8, 8), bool)
    one[3, 3] = True
    assert len(ref.word_rects(pack_bits(one), 8, 8, min_area=0)) == 0


def test_db_boxes_oracle_steps():
    """oracle_db_boxes against its steps restated in numpy on the oracle's own pieces
    (word_rects without expand, db_score): the size and score filters, unclip, page scaling and
    the reading order of src/ppdet.rs:87-132."""
    from _helpers import db_map

    prob = db_map(1)
    h, w = prob.shape
    tp = np.float32([3.4647, 3.4375])
    got = ref.db_boxes(prob, tp, 0.3)
    f = np.float32
    rects = ref.word_rects(pack_bits(prob > f(0.3)), w, h, 0.0, 0.0, -np.inf)
    keep = []
    for r in rects:
        if min(r[4], r[5]) < f(3) or ref.db_scores(prob, r[None])[0] < f(0.45):
            continue
        d = f(r[4] * r[5] * f(1.4)) / max(f(2) * f(r[4] + r[5]), f(1e-6))
        nw, nh = f(r[4] + f(2) * d), f(r[5] + f(2) * d)
        if min(nw, nh) < f(5):
            continue
        s = f(f(tp[0] + tp[1]) / f(2))
        keep.append([r[0] * tp[0], r[1] * tp[1], r[2], r[3], nw * s, nh * s])
    keep = np.float32(keep)
    assert 30 < len(keep) < len(rects)

    def bounds(r):
        hw, hh = r[4] / f(2), r[5] / f(2)
        xs = [r[0] + f(sa) * hh * r[2] + f(sb) * hw * -r[3] for sa in (-1, 1) for sb in (-1, 1)]
        ys = [r[1] + f(sa) * hh * r[3] + f(sb) * hw * r[2] for sa in (-1, 1) for sb in (-1, 1)]
        return min(xs), min(ys)

    order = sorted(range(len(keep)), key=lambda i: bounds(keep[i])[1])
    for i in range(len(order)):
        j = i
        while j > 0:
            (la, ta), (lb, tb) = bounds(keep[order[j - 1]]), bounds(keep[order[j]])
            if abs(tb - ta) < 10 and lb < la:
                order[j - 1], order[j] = order[j], order[j - 1]
                j -= 1
            else:
                break
    np.testing.assert_array_equal(got, keep[order])
