"""Per-operator parity of the CUDA path against the CPU oracle, through the C ABI, on small
and odd shapes (non-multiples of the tiles, one input channel, strides (2, 1), asymmetric pads,
channel slices).  Each case is a tiny ONNX-style graph run by NdGraph (src/nd.rs) or by the
ocrs Graph executor behind Detector::detect (src/gpu.rs)."""
import numpy as np
import pytest

import wocr
from oracle import ref
from wocr import synth
from wocr.synth import _Builder

from _helpers import argmax_parity, max_ties

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(7)


def rnd(*s):
    return RNG.standard_normal(s).astype(np.float32)


def close(a, b, tol=2e-4):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    assert a.shape == b.shape, (a.shape, b.shape)
    scale = max(1.0, float(np.abs(b).max()))
    err = float(np.abs(a - b).max()) / scale
    assert err < tol, f"max relative error {err}"


def run_nd(gpu, m, x, stop=False):
    g = wocr.NdGraph(gpu, m, stop)
    try:
        return g.run(x)
    finally:
        g.close()


@pytest.mark.parametrize("cin,cout,k,stride,pads,group,act", [
    (3, 32, 3, (2, 2), [1, 1, 1, 1], 1, "relu"),
    (16, 24, 3, (1, 1), [1, 1, 1, 1], 1, None),
    (32, 64, 1, (1, 1), [0, 0, 0, 0], 1, "relu"),
    (64, 64, 3, (2, 2), [1, 1, 1, 1], 64, "relu"),     # depthwise s2
    (24, 24, 3, (2, 1), [1, 1, 1, 1], 24, None),       # depthwise (2, 1)
    (5, 7, 3, (2, 2), [0, 0, 1, 1], 1, None),          # asymmetric pads, generic K decode
    (8, 130, 3, (1, 1), [1, 1, 1, 1], 1, "relu"),      # N not a multiple of the tile
    (16, 1, 1, (1, 1), [0, 0, 0, 0], 1, None),         # narrow 1 x 1 head: pointwise kernel
    (13, 5, 1, (1, 1), [0, 0, 0, 0], 1, "relu"),       # pointwise, cin not a multiple of 4
])
def test_conv(gpu, cin, cout, k, stride, pads, group, act):
    b = _Builder(3)
    y = b.conv("x", cin, cout, k, stride=stride, pads=pads, group=group)
    if act:
        y = b.op("Relu", [y])
    m = b.model("x", y)
    x = rnd(2, cin, 19, 37)
    close(run_nd(gpu, m, x), ref.run_onnx(m, x))


def test_conv_fusions(gpu):
    """bias Add + GELU chain + residual Add, and the squeeze-excitation input scale."""
    b = _Builder(4)
    c = b.conv("x", 16, 16, 3, bias=False)
    c = b.op("Add", [c, b.w("B", RNG.standard_normal((1, 16, 1, 1)))])
    g = b.gelu(c)
    r = b.op("Add", [g, "x"])
    s = b.se(r, 16)
    y = b.op("Relu", [b.conv(s, 16, 32, 1, pads=[0, 0, 0, 0])])
    m = b.model("x", y)
    x = rnd(2, 16, 12, 20)
    close(run_nd(gpu, m, x), ref.run_onnx(m, x))


def test_convt_batchnorm_resize_concat(gpu):
    b = _Builder(5)
    t = b.op("Relu", [b.batchnorm(b.convt("x", 12, 8, 2, 2), 8)])    # ConvT GEMM path + BN
    u = b.op("Sigmoid", [b.convt("x", 12, 4, 3, 2)])                 # general ConvT (gather)
    u = b.op("Slice", [u, b.i("s", [0, 0]), b.i("e", [14, 26]), b.i("a", [2, 3])])
    sc = b.w("scales", np.array([1, 1, 2, 2], np.float32))
    r = b.op("Resize", ["x", "", sc], {"mode": "nearest", "coordinate_transformation_mode": "asymmetric"})
    r = b.conv(r, 12, 4, 1, pads=[0, 0, 0, 0])
    y = b.op("Concat", [t, u, r], {"axis": 1})
    y = b.op("MaxPool", [y], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]})
    m = b.model("x", y)
    x = rnd(1, 12, 7, 13)
    close(run_nd(gpu, m, x), ref.run_onnx(m, x))


@pytest.mark.parametrize("cin,cout", [(32, 16), (64, 32), (24, 48)])
def test_convt_scatter_full_taps(gpu, cin, cout):
    """ConvTranspose k == s == 2 as one GEMM whose N tile spans all four taps; the scatter
    epilogue stores 16 contiguous channels per chunk (cout a multiple of 16)."""
    b = _Builder(8)
    y = b.op("Relu", [b.convt("x", cin, cout, 2, 2)])
    m = b.model("x", y)
    x = rnd(2, cin, 9, 23)
    close(run_nd(gpu, m, x), ref.run_onnx(m, x))


def test_svtr_block(gpu):
    """LayerNorm chain, Linear + bias, attention via Reshape/Transpose/Slice/MatMul/Softmax,
    Linear + SiLU; the stop before the final Softmax."""
    from wocr.synth import _svtr_block
    b = _Builder(6)
    x = _svtr_block(b, "x")
    y = b.layer_norm(x, 120)
    y = b.linear(y, 120, 37)
    y = b.op("Softmax", [y], {"axis": 2})
    m = b.model("x", y)
    x = rnd(3, 11, 120)
    close(run_nd(gpu, m, x), ref.run_onnx(m, x))
    close(run_nd(gpu, m, x, stop=True), ref.run_onnx(m, x, stop_before_softmax=True))


def test_linear_pre_split_rows(gpu, monkeypatch):
    """A linear layer whose input rows are read by many N tiles (18,709 classes: 74 tiles of 256)
    splits them once into bf16 hi / lo rows that the TMA engine loads; its results equal those of
    the producer warps' own split (WOCR_NO_A_TMA) exactly: the output, and the fused arg-max's
    classes, maxima and log-sum-exp.  The output also matches the oracle's fp32 GEMM."""
    b = _Builder(15)
    m = b.model("x", b.linear("x", 120, 18709))
    x = rnd(1, 300, 120)
    g = wocr.NdGraph(gpu, m)
    try:
        monkeypatch.setenv("WOCR_NO_GRAPH", "1")  # every call launches, reading the variable
        out = g.run(x)
        best, mx, lse, shape = g.argmax(x)
        monkeypatch.setenv("WOCR_NO_A_TMA", "1")
        out2 = g.run(x)
        best2, mx2, lse2, shape2 = g.argmax(x)
    finally:
        g.close()
    assert shape == shape2 == (1, 300, 18709)
    assert np.array_equal(out, out2)
    assert np.array_equal(best, best2) and np.array_equal(mx, mx2) and np.array_equal(lse, lse2)
    close(out, ref.run_onnx(m, x), tol=5e-5)


@pytest.mark.parametrize("classes", [37, 700, 1031])
def test_linear_argmax_fused(gpu, classes, monkeypatch):
    """A final linear layer with the row arg-max in its epilogue (per N tile partials merged):
    one tile, several tiles, a last partial tile; equals the oracle's arg-max, maximum and
    log-sum-exp, and the unfused path's arg-max and maximum exactly."""
    b = _Builder(14)
    y = b.linear(b.layer_norm("x", 120), 120, classes)
    m = b.model("x", y)
    x = rnd(3, 50, 120)
    g = wocr.NdGraph(gpu, m)
    try:
        best, mx, lse, shape = g.argmax(x)
        # without the log-sum-exp (the epilogue skips the exponentials): the same classes and
        # maxima, on the recorded first call and on the graph replay
        for _ in range(2):
            nb, nmx, nlse, nshape = g.argmax(x, lse=False)
            assert nlse is None and nshape == shape
            assert (nb == best).all() and (nmx == mx).all()
        monkeypatch.setenv("WOCR_UNFUSED_ARGMAX", "1")
        monkeypatch.setenv("WOCR_NO_GRAPH", "1")
        ub, umx, ulse, ushape = g.argmax(x)
    finally:
        g.close()
    assert shape == ushape == (3, 50, classes)
    assert (best == ub).all() and (mx == umx).all()
    assert np.abs(lse - ulse).max() < 1e-4
    logits = ref.run_onnx(m, x).reshape(-1, classes)
    bad, ties = argmax_parity(best, logits)
    assert bad == 0
    assert ties <= max_ties(len(best)), f"{ties} near-tie steps of {len(best)}"
    _, rmx, _, rlse = ref.argmax(logits)
    assert np.abs(mx - rmx).max() < 1e-4 and np.abs(lse - rlse).max() < 1e-4


def test_int_shape_ops_and_pools(gpu):
    b = _Builder(8)
    p = b.op("AveragePool", ["x"], {"kernel_shape": [3, 3], "strides": [2, 2], "auto_pad": "SAME_UPPER"})
    p = b.op("HardSigmoid", [p], {"alpha": 0.3, "beta": 0.4})
    gp = b.op("GlobalAveragePool", [p])
    shp = b.op("Shape", [p])
    nb = b.op("Unsqueeze", [b.op("Gather", [shp, b.i("i", [0])]), b.i("ax", [0])])
    tgt = b.op("Concat", [nb, b.i("rest", [-1])], {"axis": 0})
    flat = b.op("Reshape", [p, tgt])
    red = b.op("ReduceMean", [flat], {"axes": [-1], "keepdims": 0})
    y = b.op("Mul", [b.op("Reshape", [gp, b.i("s2", [0, -1])]), b.op("Unsqueeze", [red, b.i("a2", [1])])])
    y = b.op("Pow", [b.op("Sub", [y, b.scalar("c", 0.1)]), b.scalar("two", 2.0)])
    y = b.op("Div", [b.op("Sqrt", [y]), b.scalar("d", 3.0)])
    m = b.model("x", y)
    x = rnd(2, 6, 9, 14)
    close(run_nd(gpu, m, x), ref.run_onnx(m, x))


def test_graph_executor_ops(gpu):
    """The ocrs executor: Direct conv + fused MaxPool, dense convs, standalone MaxPool, zero Pad,
    Slice, ConvTranspose + Relu, channel Concat, standalone Sigmoid."""
    b = _Builder(9)
    d = b.maxpool(b.conv_relu("image", 1, 16, 3), 2, 2)
    c = b.conv_relu(d, 16, 32, 3)
    p = b.maxpool(c, 2, 2)
    p = b.op("Pad", [p, b.i("pads", [0] * 8)])
    u = b.op("Relu", [b.convt(p, 32, 16, 2, 2)])
    u = b.op("Slice", [u, b.i("st", [0]), b.i("en", [16]), b.i("ax", [1])])
    y = b.op("Concat", [u, d], {"axis": 1})
    y = b.op("Sigmoid", [b.conv(y, 32, 1, 1, pads=[0, 0, 0, 0])])
    m = b.model("image", y)
    x = rnd(1, 1, 44, 60)
    det = wocr.Detector(gpu, m)
    try:
        close(det.detect(x), ref.run_onnx(m, x)[0, 0])
    finally:
        det.close()


def _det_parity(gpu, m, x):
    det = wocr.Detector(gpu, m)
    try:
        close(det.detect(x), ref.run_onnx(m, x)[0, 0])
    finally:
        det.close()


def test_graph_split_activations(gpu):
    """Values between the convolutions stored split (bf16 hi | lo) and read by the tap
    convolution: 3 x 3 and 5 x 5 kernels, a partial 16-channel chunk (24 channels) and a
    partial 32-channel chunk (40), N below one column chunk (8), the ConvTranspose scatter,
    a split Concat, split MaxPool, the pointwise head; a cin = 8 conv takes the fp32 path."""
    b = _Builder(12)
    d = b.maxpool(b.conv_relu("image", 1, 16, 3), 2, 2)                  # 26 x 36
    a = b.conv_relu(d, 16, 24, 3)
    a2 = b.op("Relu", [b.conv(a, 24, 32, 5, pads=[2, 2, 2, 2])])
    p = b.maxpool(a2, 2, 2)                                              # 13 x 18
    u = b.op("Relu", [b.convt(p, 32, 16, 2, 2)])                         # 26 x 36
    y = b.op("Concat", [u, a], {"axis": 1})                              # 40 channels
    e = b.conv_relu(y, 40, 8, 3)
    f = b.conv_relu(e, 8, 16, 1)
    g = b.conv_relu(f, 16, 20, 3)
    out = b.op("Sigmoid", [b.conv(g, 20, 1, 1, pads=[0, 0, 0, 0])])
    m = b.model("image", out)
    _det_parity(gpu, m, rnd(1, 1, 52, 72))
    _det_parity(gpu, m, rnd(1, 1, 36, 44))


def test_graph_split_fallbacks(gpu):
    """Split values whose slices break the TMA alignment (a Concat of 16 + 12 + 24 channels puts
    the 24-channel part at channel 28) and a ConvTranspose with cout % 16 != 0 (per-channel
    scatter stores): these run through the fp32 conversions."""
    b = _Builder(13)
    d = b.maxpool(b.conv_relu("image", 1, 16, 3), 2, 2)
    a = b.conv_relu(d, 16, 24, 3)
    p = b.maxpool(b.conv_relu(a, 24, 32, 3), 2, 2)
    u = b.op("Relu", [b.convt(p, 32, 16, 2, 2)])
    v = b.op("Relu", [b.convt(p, 32, 12, 2, 2)])
    y = b.op("Concat", [u, v, a], {"axis": 1})                           # 52 channels
    g = b.conv_relu(y, 52, 16, 3)
    out = b.op("Sigmoid", [b.conv(g, 16, 1, 1, pads=[0, 0, 0, 0])])
    m = b.model("image", out)
    _det_parity(gpu, m, rnd(1, 1, 40, 56))


@pytest.mark.parametrize("hw", [(52, 72), (36, 100), (404, 700)])
@pytest.mark.parametrize("rows", [True, False])
def test_graph_narrow_3x3_layers(gpu, hw, rows, monkeypatch):
    """The narrow 3 x 3 layers (<= 32 output channels, <= 64 input channels) of a small U-Net,
    by the row kernel (kernel columns stacked along N, the column sums gathered by shuffles)
    and, with WOCR_NO_ROWS, by the per-tap kernel: 16 -> 16 with a fused MaxPool, 16 -> 32,
    32 -> 32 with a fused MaxPool, 64 -> 32 and 32 -> 16 behind split Concats.  Widths that are
    not multiples of the 14-column tile; 404 x 700 (283 K pixels) takes the two-block tiles."""
    if not rows:
        monkeypatch.setenv("WOCR_NO_ROWS", "1")
    b = _Builder(21)
    x0 = b.conv_relu("image", 1, 16, 3)
    a0 = b.conv_relu(x0, 16, 16, 3)
    a1 = b.conv_relu(b.maxpool(a0, 2, 2), 16, 32, 3)
    a1b = b.conv_relu(a1, 32, 32, 3)
    a2 = b.conv_relu(b.maxpool(a1b, 2, 2), 32, 64, 3)
    u1 = b.op("Relu", [b.convt(a2, 64, 32, 2, 2)])
    d1 = b.conv_relu(b.op("Concat", [u1, a1b], {"axis": 1}), 64, 32, 3)
    u0 = b.op("Relu", [b.convt(d1, 32, 16, 2, 2)])
    d0 = b.conv_relu(b.op("Concat", [u0, a0], {"axis": 1}), 32, 16, 3)
    out = b.op("Sigmoid", [b.conv(d0, 16, 1, 1, pads=[0, 0, 0, 0])])
    m = b.model("image", out)
    _det_parity(gpu, m, rnd(1, 1, *hw))


def test_unsupported_and_shape_errors(gpu):
    b = _Builder(10)
    y = b.op("LeakyRelu", ["x"])
    with pytest.raises(wocr.WocrError) as e:
        run_nd(gpu, b.model("x", y), rnd(1, 2, 3, 4))
    assert e.value.code == 2 and "unsupported op LeakyRelu" in e.value.message
    b = _Builder(11)
    y = b.conv("x", 4, 4, 3)
    with pytest.raises(wocr.WocrError) as e:
        run_nd(gpu, b.model("x", y), rnd(1, 3, 8, 8))           # 3 channels into a 4-channel conv
    assert e.value.code == 3
    b = _Builder(12)
    y = b.conv("image", 2, 4, 3, group=2)                           # grouped, not depthwise
    with pytest.raises(wocr.WocrError) as e:
        wocr.Detector(gpu, b.model("image", y))
    assert e.value.code == 2


@pytest.mark.parametrize("m,k,n", [(1, 120, 97), (300, 120, 360), (257, 512, 1536), (130, 120, 18709),
                                   (64, 240, 120), (7, 256, 1536)])
def test_linear_shapes(gpu, m, k, n):
    """MatMul with a constant [K, N] weight + bias (the tensor-core GEMM with K padded to 64 and
    N over several tiles), against the oracle's fp32 GEMM."""
    b = _Builder(20 + n)
    y = b.linear("x", k, n, init="he")
    mdl = b.model("x", y)
    x = rnd(m, k)
    close(run_nd(gpu, mdl, x), ref.run_onnx(mdl, x), tol=5e-5)


def test_handles_outlive_their_context():
    """Destroying the device context before the graphs made from it is safe: the context is
    released with its last handle (Python may collect them in any order)."""
    g = wocr.Gpu()
    b = _Builder(30)
    m = b.model("x", b.op("Relu", [b.conv("x", 8, 16, 3)]))
    nd = wocr.NdGraph(g, m)
    g.close()
    x = rnd(1, 8, 9, 11)
    close(nd.run(x), ref.run_onnx(m, x))
    nd.close()


def _pp_boxes(w, h, rng):
    """Line boxes of a page: ordinary lines (down- and upsampled heights), boxes on the page's
    edges and corners, a box reaching past the last row, degenerate (empty, reversed, NaN) boxes,
    fractional coordinates, and tall crops for the two-pass kernels (383 and 384 rows, the whole
    page)."""
    boxes = [[rng.uniform(0, w - 800), y, 0, 0] for y in rng.uniform(0, h - 120, 20)]
    for b in boxes:
        b[2] = b[0] + rng.uniform(30, 800)
        b[3] = b[1] + rng.uniform(12, 110)
    boxes += [[0, 0, 37, 21], [w - 13, h - 9, w + 40, h + 40], [w, 100, w, 140], [500, h - 3, 900, h + 50],
              [300, 400, 200, 380], [float("nan"), 10, 60, 40], [10.7, 20.2, 1500.9, 20.9], [0, 0, w, 60],
              [100, 200, 110, 1900], [40, 500, 900, 883], [40, 500, 900, 884], [0, 0, w, h],
              [50, 100, 2400, 3000]]
    return np.array(boxes, np.float32)


def test_pp_lines_bit_exact(gpu):
    """Recognition line batches cut on the device (ppocr.rs line_input + ocr-bench.rs pp_batches):
    the layout (order, batch sizes and widths) and every value equal the oracle's; 19 lines per
    batch leaves a partial last batch."""
    import torch

    w, h = 2550, 3300
    page = synth.page(7, w, h)
    rects = _pp_boxes(w, h, np.random.default_rng(3))
    order, batches, total = gpu.pp_lines(0, w, h, rects, per_batch=19)
    rb, rorder = ref.pp_batches(page, rects, per=19)
    assert order == rorder
    assert batches == [(n, wd) for _, n, wd in rb]
    d_page = torch.from_numpy(page).cuda()
    d_out = torch.full((total,), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    gpu.pp_lines(d_page.data_ptr(), w, h, rects, per_batch=19, d_out=d_out.data_ptr(), cap=total)
    got = d_out.cpu().numpy()
    want = np.concatenate([b.ravel() for b, _, _ in rb])
    assert got.shape == want.shape
    np.testing.assert_array_equal(got, want)
    with pytest.raises(wocr.WocrError):
        gpu.pp_lines(d_page.data_ptr(), w, h, rects, per_batch=19, d_out=d_out.data_ptr(), cap=total - 1)
