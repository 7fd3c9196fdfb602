"""Seeded synthetic models and inputs for the benchmark configurations.

The real ocrs and PP-OCRv6 `.onnx` files are not available (they are downloaded over the
network by the reference's `scripts/fetch-models.sh`), so every model here is a random-init
graph of the published architecture family, written node by node the way an ONNX exporter
writes it, and restricted to the ops and attribute forms the reference executors accept
(`src/gpu.rs:1104-1240` for the ocrs graphs, `src/nd.rs:505-817, 834-1195` for PP-OCR).

All generators are deterministic functions of their seed (numpy PCG64), so the CUDA path,
the CPU oracle and the CPU baseline see identical bytes.

Configurations (numbering of the benchmark configs):
  0  ocrs recognition: conv trunk 64 -> 1 rows, 2 bidirectional GRU layers (hidden 256),
     linear 512 -> 97.  Weights: conv He-normal, GRU U(+-1/16), seed 0.
  1  ocrs detection U-Net (16/32/64/128 channels, 3 MaxPool levels, ConvTranspose decoder
     with skip Concat, 1x1 head + Sigmoid).  He-normal, seed 1.
  3  PP-OCRv6-style recognition: stride-2 conv + depthwise-separable trunk (one HardSigmoid
     squeeze-excitation block), SVTR neck (2 blocks, dim 120, 8 heads, MLP 240), LayerNorm,
     CTC head 120 -> 18,709.  Raw weights trunc-normal(std 0.02, +-2 std), seed 2; the conv
     trunk carries folded BatchNorm whose calibrated scale restores unit activation variance.
  4  PP-OCRv6-style DB detector: depthwise-separable backbone to 1/32, FPN (1x1 laterals,
     nearest x2 top-down adds, 3x3 smoothing, nearest upsample + Concat), DB head (conv, BN,
     ReLU, 2x ConvTranspose, Sigmoid).  He-normal, seed 3.
"""
from __future__ import annotations

import math
from typing import Dict, List, Sequence, Tuple

import numpy as np

from .model import Model, Node

# ocrs' alphabet (`src/bin/ocr-bench.rs:31`): class c > 0 is ALPHABET[c - 1]; class 0 is blank.
OCRS_ALPHABET = (" 0123456789!\"#$%&'()*+,-./:;<=>?@[\\]^_`{|}~EABCDEFGHIJKLMNOPQRSTUVWXYZ"
                 "abcdefghijklmnopqrstuvwxyz")
OCRS_CLASSES = 97
PP_CLASSES = 18709
OCRS_BLACK = -0.5          # ocrs line-image padding value (`src/bin/ocr-bench.rs:32`)
DET_H, DET_W = 800, 600    # ocrs detection model input (`src/gpu.rs:1394`)
PP_HEIGHT = 48             # PP-OCR line height (`src/ppocr.rs:39`)


class _Builder:
    """Appends ONNX-style nodes and initializers with unique value names."""

    def __init__(self, seed: int):
        self.rng = np.random.default_rng(seed)
        self.nodes: List[Node] = []
        self.weights: Dict[str, np.ndarray] = {}
        self.ints: Dict[str, np.ndarray] = {}
        self.k = 0

    def name(self, prefix: str) -> str:
        self.k += 1
        return f"{prefix}_{self.k}"

    def w(self, prefix: str, arr) -> str:
        n = self.name(prefix)
        self.weights[n] = np.ascontiguousarray(arr, dtype=np.float32)
        return n

    def i(self, prefix: str, vals) -> str:
        n = self.name(prefix)
        self.ints[n] = np.asarray(vals, dtype=np.int64).reshape(-1)
        return n

    def op(self, op: str, inputs: Sequence[str], attrs=None) -> str:
        out = self.name(op.lower())
        self.nodes.append(Node(op, list(inputs), [out], dict(attrs or {})))
        return out

    # --- initialisers ---------------------------------------------------------------
    def he(self, shape, fan_in):
        return self.rng.normal(0.0, math.sqrt(2.0 / fan_in), size=shape)

    def trunc_normal(self, shape, std=0.02):
        """Normal(0, std) truncated at +-2 std by rejection."""
        out = self.rng.normal(0.0, std, size=shape)
        bad = np.abs(out) > 2 * std
        while bad.any():
            out[bad] = self.rng.normal(0.0, std, size=int(bad.sum()))
            bad = np.abs(out) > 2 * std
        return out

    def uniform(self, shape, bound):
        return self.rng.uniform(-bound, bound, size=shape)

    # --- layers ---------------------------------------------------------------------
    def conv(self, x, cin, cout, k, stride=(1, 1), pads=None, group=1, bias=True, init="he",
             weight_scale=1.0):
        kh, kw = (k, k) if isinstance(k, int) else k
        if pads is None:
            pads = [kh // 2, kw // 2, kh // 2, kw // 2]
        cin_g = cin // group
        fan_in = cin_g * kh * kw
        shape = (cout, cin_g, kh, kw)
        if init == "he":
            wv = self.he(shape, fan_in)
        elif init == "tn_bn":
            # trunc-normal raw weights with folded, calibrated BatchNorm: scale restores He gain
            wv = self.trunc_normal(shape) * (math.sqrt(2.0 / fan_in) / 0.02)
        else:
            raise ValueError(init)
        wv = wv * weight_scale
        ins = [x, self.w("W", wv)]
        if bias:
            ins.append(self.w("B", self.rng.normal(0.0, 0.05, size=(cout,))))
        attrs = {"kernel_shape": [kh, kw], "pads": list(pads), "strides": list(stride),
                 "dilations": [1, 1]}
        if group != 1:
            attrs["group"] = group
        return self.op("Conv", ins, attrs)

    def conv_relu(self, x, cin, cout, k, **kw):
        return self.op("Relu", [self.conv(x, cin, cout, k, **kw)])

    def maxpool(self, x, kh, kw):
        return self.op("MaxPool", [x], {"kernel_shape": [kh, kw], "strides": [kh, kw]})

    def convt(self, x, cin, cout, k, s, bias=True):
        wv = self.he((cin, cout, k, k), cin)
        ins = [x, self.w("Wt", wv)]
        if bias:
            ins.append(self.w("Bt", self.rng.normal(0.0, 0.05, size=(cout,))))
        return self.op("ConvTranspose", ins, {"kernel_shape": [k, k], "strides": [s, s]})

    def batchnorm(self, x, c):
        g = self.w("bn_g", 1.0 + 0.1 * self.rng.standard_normal(c))
        b = self.w("bn_b", 0.1 * self.rng.standard_normal(c))
        m = self.w("bn_m", 0.1 * self.rng.standard_normal(c))
        v = self.w("bn_v", self.rng.uniform(0.5, 1.5, size=c))
        return self.op("BatchNormalization", [x, g, b, m, v], {"epsilon": 1e-5})

    def scalar(self, prefix, v):
        return self.w(prefix, np.array([v], np.float32))

    def linear(self, x, k, n, init="tn"):
        if init == "tn":
            wv = self.trunc_normal((k, n))
        else:
            wv = self.he((k, n), k)
        y = self.op("MatMul", [x, self.w("Wl", wv)])
        bias = np.zeros(n) if init == "tn" else self.rng.normal(0.0, 0.05, size=n)
        return self.op("Add", [y, self.w("Bl", bias)])

    def layer_norm(self, x, dim):
        """The exporter's 9-node LayerNorm chain (`src/nd.rs:583-611` fuses exactly this)."""
        mean = self.op("ReduceMean", [x], {"axes": [-1]})
        d = self.op("Sub", [x, mean])
        p = self.op("Pow", [d, self.scalar("two", 2.0)])
        var = self.op("ReduceMean", [p], {"axes": [-1]})
        a = self.op("Add", [var, self.scalar("eps", 1e-6)])
        s = self.op("Sqrt", [a])
        q = self.op("Div", [d, s])
        g = self.op("Mul", [q, self.w("ln_g", 1.0 + self.trunc_normal((dim,)))])
        return self.op("Add", [g, self.w("ln_b", self.trunc_normal((dim,)))])

    def gelu(self, x):
        """The exporter's GELU chain x * (erf(x / sqrt 2) + 1) * 0.5 (`src/nd.rs:676-700`)."""
        d = self.op("Div", [x, self.scalar("sqrt2", math.sqrt(2.0))])
        e = self.op("Erf", [d])
        a = self.op("Add", [e, self.scalar("one", 1.0)])
        m = self.op("Mul", [x, a])
        return self.op("Mul", [m, self.scalar("half", 0.5)])

    def silu(self, x):
        s = self.op("Sigmoid", [x])
        return self.op("Mul", [x, s])

    def se(self, x, c, r=4, init="he"):
        """Squeeze-excitation gated by HardSigmoid: Mul(x, gate) (`src/nd.rs:552-571`)."""
        g = self.op("GlobalAveragePool", [x])
        g = self.conv_relu(g, c, c // r, 1, pads=[0, 0, 0, 0], init=init)
        g = self.conv(g, c // r, c, 1, pads=[0, 0, 0, 0], init=init)
        g = self.op("HardSigmoid", [g], {"alpha": 0.2, "beta": 0.5})
        return self.op("Mul", [x, g])

    def model(self, inp, out) -> Model:
        return Model(self.nodes, self.weights, self.ints, inp, out)


# ---------------------------------------------------------------------------------------
# config 0: ocrs recognition
# ---------------------------------------------------------------------------------------
def ocrs_rec_model(seed: int = 0) -> Model:
    b = _Builder(seed)
    x = "line"
    x = b.maxpool(b.conv_relu(x, 1, 32, 3), 2, 2)        # Direct conv + fused MaxPool
    x = b.maxpool(b.conv_relu(x, 32, 64, 3), 2, 2)
    x = b.conv_relu(x, 64, 128, 3)
    x = b.maxpool(b.conv_relu(x, 128, 128, 3), 2, 1)
    x = b.conv_relu(x, 128, 256, 3)
    x = b.maxpool(b.conv_relu(x, 256, 256, 3), 2, 1)       # [n, 256, 4, W/4]
    x = b.op("AveragePool", [x], {"kernel_shape": [4, 1], "strides": [4, 1]})
    x = b.op("Squeeze", [x, b.i("axes", [2])])             # [n, 256, T]
    x = b.op("Transpose", [x], {"perm": [2, 0, 1]})        # [T, n, 256]
    bound = 1.0 / 16.0
    for inp in (256, 512):
        W = b.w("gru_W", b.uniform((2, 768, inp), bound))
        R = b.w("gru_R", b.uniform((2, 768, 256), bound))
        B = b.w("gru_B", b.uniform((2, 1536), bound))
        y = b.op("GRU", [x, W, R, B], {"hidden_size": 256, "direction": "bidirectional",
                                       "linear_before_reset": 1})  # [T, 2, n, 256]
        y = b.op("Transpose", [y], {"perm": [0, 2, 1, 3]})         # [T, n, 2, 256]
        x = b.op("Reshape", [y, b.i("shape", [0, 0, 512])])        # [T, n, 512]
    out = b.linear(x, 512, OCRS_CLASSES, init="he")                # [T, n, 97]
    return b.model("line", out)


# ---------------------------------------------------------------------------------------
# config 1: ocrs detection U-Net
# ---------------------------------------------------------------------------------------
def ocrs_det_model(seed: int = 1) -> Model:
    b = _Builder(seed)
    x = "image"
    chans = [16, 32, 64, 128]
    skips = []
    cin = 1
    for lvl, c in enumerate(chans):
        x = b.conv_relu(x, cin, c, 3)
        x = b.conv_relu(x, c, c, 3)
        cin = c
        if lvl < 3:
            skips.append(x)
            x = b.maxpool(x, 2, 2)
    for lvl in (2, 1, 0):
        c = chans[lvl]
        x = b.op("Relu", [b.convt(x, cin, c, 2, 2)])
        x = b.op("Concat", [x, skips[lvl]], {"axis": 1})
        x = b.conv_relu(x, 2 * c, c, 3)
        x = b.conv_relu(x, c, c, 3)
        cin = c
    # a zero Pad (`src/gpu.rs:1218-1224` lowers it to Identity)
    x = b.op("Pad", [x, b.i("pads", [0] * 8)], {"mode": "constant"})
    out = b.op("Sigmoid", [b.conv(x, 16, 1, 1, pads=[0, 0, 0, 0], weight_scale=4.0)])
    return b.model("image", out)


def ocrs_ink_det_model(gain: float = 10.0, bias: float = -1.0) -> Model:
    """A hand-set stand-in for the trained ocrs detector, for the page pipeline's tests and its
    secondary measurement (not the config's random-init model): darkness (a 1 x 1 conv, 0.5 - x,
    so white and the convolution's zero padding are both 0), a 5 x 5 conv whose middle three rows
    sum it (the outer rows zero), and a sigmoid.  On page(...), resized to 800 x 600, a glyph gap
    (1-4 px there) stays above the 0.5 threshold and a word gap (6 px or more) falls below it, so
    the mask marks words and a page has its 36 text lines."""
    b = _Builder(0)
    ins = ["image", b.w("W", -np.ones((1, 1, 1, 1))), b.w("B", np.full(1, 0.5))]
    d = b.op("Conv", ins, {"kernel_shape": [1, 1], "pads": [0, 0, 0, 0], "strides": [1, 1], "dilations": [1, 1]})
    wt = np.zeros((1, 1, 5, 5))
    wt[0, 0, 1:4, :] = gain / 15.0
    ins = [d, b.w("W", wt), b.w("B", np.full(1, bias))]
    c = b.op("Conv", ins, {"kernel_shape": [5, 5], "pads": [2, 2, 2, 2], "strides": [1, 1], "dilations": [1, 1]})
    return b.model("image", b.op("Sigmoid", [c]))


# ---------------------------------------------------------------------------------------
# config 3: PP-OCRv6-style recognition (trunk + SVTR neck + CTC head)
# ---------------------------------------------------------------------------------------
def _svtr_block(b: _Builder, x, dim=120, heads=8, mlp=240):
    hd = dim // heads
    y = b.layer_norm(x, dim)
    qkv = b.linear(y, dim, 3 * dim)                                      # [n, T, 360]
    qkv = b.op("Reshape", [qkv, b.i("shape", [0, -1, 3, heads, hd])])     # [n, T, 3, 8, 15]
    qkv = b.op("Transpose", [qkv], {"perm": [2, 0, 3, 1, 4]})            # [3, n, 8, T, 15]
    parts = []
    for s in range(3):
        p = b.op("Slice", [qkv, b.i("starts", [s]), b.i("ends", [s + 1]), b.i("axes", [0])])
        parts.append(b.op("Squeeze", [p, b.i("axes", [0])]))             # [n, 8, T, 15]
    q, k, v = parts
    q = b.op("Mul", [q, b.scalar("qk_scale", hd ** -0.5)])
    kt = b.op("Transpose", [k], {"perm": [0, 1, 3, 2]})                  # [n, 8, 15, T]
    att = b.op("Softmax", [b.op("MatMul", [q, kt])], {"axis": -1})       # [n, 8, T, T]
    o = b.op("MatMul", [att, v])                                         # [n, 8, T, 15]
    o = b.op("Transpose", [o], {"perm": [0, 2, 1, 3]})                   # [n, T, 8, 15]
    o = b.op("Reshape", [o, b.i("shape", [0, 0, dim])])
    x = b.op("Add", [x, b.linear(o, dim, dim)])
    y = b.layer_norm(x, dim)
    y = b.silu(b.linear(y, dim, mlp))                                    # MatMul + bias + SiLU
    return b.op("Add", [x, b.linear(y, mlp, dim)])


def pp_rec_model(seed: int = 2, classes: int = PP_CLASSES) -> Model:
    b = _Builder(seed)
    tn = dict(init="tn_bn")
    x = "x"                                                              # [n, 3, 48, W]
    x = b.conv_relu(x, 3, 32, 3, stride=(2, 2), **tn)                    # [32, 24, W/2]

    def ds(x, cin, cout, stride, se=False):
        x = b.conv_relu(x, cin, cin, 3, stride=stride, group=cin, **tn)  # depthwise
        if se:
            x = b.se(x, cin, init="he")
        return b.conv_relu(x, cin, cout, 1, pads=[0, 0, 0, 0], **tn)     # pointwise

    x = ds(x, 32, 64, (1, 1))                                            # [64, 24, W/2]
    x = ds(x, 64, 128, (2, 2))                                           # [128, 12, W/4]
    x = ds(x, 128, 256, (2, 2), se=True)                                 # [256, 6, W/8]
    x = ds(x, 256, 256, (2, 1))                                          # [256, 3, W/8]
    x = b.maxpool(x, 3, 1)                                               # [256, 1, W/8]
    r = b.conv_relu(x, 256, 256, 1, pads=[0, 0, 0, 0], **tn)
    x = b.op("Add", [r, x])                                              # fused residual
    c = b.conv(x, 256, 120, 1, pads=[0, 0, 0, 0], bias=False, **tn)
    c = b.op("Add", [c, b.w("B", b.rng.normal(0.0, 0.05, size=(1, 120, 1, 1)))])
    x = b.gelu(c)                                                        # [n, 120, 1, T]
    # [n, 120, 1, T] -> [n, 120, T] with the batch size taken from Shape (integer subgraph)
    shp = b.op("Shape", [x])
    nb = b.op("Gather", [shp, b.i("idx", [0])])
    nb = b.op("Unsqueeze", [nb, b.i("axes", [0])])
    tgt = b.op("Concat", [nb, b.i("rest", [120, -1])], {"axis": 0})
    x = b.op("Reshape", [x, tgt])
    x = b.op("Transpose", [x], {"perm": [0, 2, 1]})                      # [n, T, 120]
    for _ in range(2):
        x = _svtr_block(b, x)
    x = b.layer_norm(x, 120)
    logits = b.linear(x, 120, classes)                                   # [n, T, classes]
    out = b.op("Softmax", [logits], {"axis": 2})
    return b.model("x", out)


# ---------------------------------------------------------------------------------------
# config 4: PP-OCRv6-style DB detector
# ---------------------------------------------------------------------------------------
def pp_ink_det_model(gain: float = 1.2, bias: float = -2.0) -> Model:
    """A hand-set stand-in for a trained DB detector, for tests of the page pipeline (not a
    benchmark model): darkness (a 1 x 1 conv summing the normalised channels, negated), a 3 x 9
    box average that joins the glyphs of a word, and a sigmoid.  On page(...) it marks word blobs,
    so a page yields hundreds of DB boxes instead of the one page-sized box of the random-init
    detector."""
    b = _Builder(0)
    ins = ["x", b.w("W", -np.ones((1, 3, 1, 1))), b.w("B", np.zeros(1))]
    d = b.op("Conv", ins, {"kernel_shape": [1, 1], "pads": [0, 0, 0, 0], "strides": [1, 1], "dilations": [1, 1]})
    ins = [d, b.w("W", np.full((1, 1, 3, 9), gain / 27.0)), b.w("B", np.full(1, bias))]
    a = b.op("Conv", ins, {"kernel_shape": [3, 9], "pads": [1, 4, 1, 4], "strides": [1, 1], "dilations": [1, 1]})
    return b.model("x", b.op("Sigmoid", [a]))


def pp_det_model(seed: int = 3) -> Model:
    b = _Builder(seed)
    x = "x"                                                              # [1, 3, H, W]
    x = b.conv_relu(x, 3, 16, 3, stride=(2, 2))                          # 1/2

    def ds(x, cin, cout, stride, se=False):
        x = b.conv_relu(x, cin, cin, 3, stride=stride, group=cin)
        if se:
            x = b.se(x, cin)
        return b.conv_relu(x, cin, cout, 1, pads=[0, 0, 0, 0])

    x = ds(x, 16, 32, (1, 1))
    c2 = ds(x, 32, 32, (2, 2))                                           # 1/4
    c3 = ds(c2, 32, 64, (2, 2))                                          # 1/8
    c4 = ds(c3, 64, 128, (2, 2), se=True)                                # 1/16
    c5 = ds(c4, 128, 256, (2, 2))                                        # 1/32
    ins = [b.conv(c, ci, 64, 1, pads=[0, 0, 0, 0], bias=False)
           for c, ci in ((c2, 32), (c3, 64), (c4, 128), (c5, 256))]

    def up(t, f):
        roi = ""
        sc = b.w("scales", np.array([1.0, 1.0, f, f], np.float32))
        return b.op("Resize", [t, roi, sc], {"mode": "nearest",
                                             "coordinate_transformation_mode": "asymmetric",
                                             "nearest_mode": "floor"})

    out4 = b.op("Add", [ins[2], up(ins[3], 2.0)])
    out3 = b.op("Add", [ins[1], up(out4, 2.0)])
    out2 = b.op("Add", [ins[0], up(out3, 2.0)])
    p5 = up(b.conv(ins[3], 64, 16, 3, bias=False), 8.0)
    p4 = up(b.conv(out4, 64, 16, 3, bias=False), 4.0)
    p3 = up(b.conv(out3, 64, 16, 3, bias=False), 2.0)
    p2 = b.conv(out2, 64, 16, 3, bias=False)
    fuse = b.op("Concat", [p5, p4, p3, p2], {"axis": 1})                 # [64, H/4, W/4]
    h = b.conv(fuse, 64, 16, 3, bias=False)
    h = b.op("Relu", [b.batchnorm(h, 16)])
    h = b.op("Relu", [b.batchnorm(b.convt(h, 16, 16, 2, 2), 16)])
    h = b.convt(h, 16, 1, 2, 2)
    out = b.op("Sigmoid", [h])
    return b.model("x", out)


# ---------------------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------------------
def _bars(rng, width: int, lo: int = 2, hi: int = 12, glo: int = 2, ghi: int = 6):
    """Column spans [x0, x1) of random-width glyph bars separated by random gaps."""
    spans = []
    x = int(rng.integers(glo, ghi + 1))
    while x < width:
        bw = int(rng.integers(lo, hi + 1))
        spans.append((x, min(width, x + bw)))
        x += bw + int(rng.integers(glo, ghi + 1))
    return spans


def ocrs_lines(seed: int = 0, n: int = 64, wmin: int = 64, wmax: int = 1024):
    """`n` ocrs line images [64, W] f32: background 0.5, vertical bars -0.5 (rows 8..56)."""
    rng = np.random.default_rng(seed + 1000)
    lines = []
    for _ in range(n):
        w = int(rng.integers(wmin // 4, wmax // 4 + 1)) * 4
        img = np.full((64, w), 0.5, np.float32)
        for x0, x1 in _bars(rng, w):
            img[8:56, x0:x1] = -0.5
        lines.append(img)
    return lines


def ocrs_batches(lines: List[np.ndarray], bucket: int = 50, per: int = 20):
    """Batch line images as `line_batches` does (`src/bin/ocr-bench.rs:365-408`): groups by
    width rounded up to `bucket`, in increasing width, chunks of at most `per` lines, padded on
    the right with -0.5.  Returns [(data [n, 1, 64, width], n, width)], line order, widths."""
    groups: Dict[int, List[int]] = {}
    for i, img in enumerate(lines):
        wb = -(-img.shape[1] // bucket) * bucket
        groups.setdefault(wb, []).append(i)
    batches, order, widths = [], [], []
    for wb in sorted(groups):
        members = groups[wb]
        for c0 in range(0, len(members), per):
            chunk = members[c0:c0 + per]
            data = np.full((len(chunk), 1, 64, wb), OCRS_BLACK, np.float32)
            for k, i in enumerate(chunk):
                data[k, 0, :, :lines[i].shape[1]] = lines[i]
                order.append(i)
                widths.append(lines[i].shape[1])
            batches.append((data, len(chunk), wb))
    return batches, order, widths


def pp_lines(seed: int = 2, n: int = 256, wmin: int = 96, wmax: int = 1280):
    """`n` PP-OCR line images [3, 48, W] in [-1, 1]: background +1, bars -1 (rows 6..42)."""
    rng = np.random.default_rng(seed + 1000)
    lines = []
    for _ in range(n):
        w = int(rng.integers(wmin // 8, wmax // 8 + 1)) * 8
        img = np.full((3, PP_HEIGHT, w), 1.0, np.float32)
        for x0, x1 in _bars(rng, w):
            img[:, 6:42, x0:x1] = -1.0
        lines.append(img)
    return lines


def pp_batches(lines: List[np.ndarray], per: int = 16):
    """Batch as `pp_batches` does by default (`src/bin/ocr-bench.rs:337-353`): sorted by width,
    cut into batches of `per`, each padded with 0 to its widest line rounded up to 8
    (`src/ppocr.rs:64-78`).  Returns [(data [n, 3, 48, width], n, width)] and the line order."""
    idx = sorted(range(len(lines)), key=lambda i: lines[i].shape[2])
    batches, order = [], []
    for c0 in range(0, len(idx), per):
        part = idx[c0:c0 + per]
        width = -(-max(lines[i].shape[2] for i in part) // 8) * 8
        data = np.zeros((len(part), 3, PP_HEIGHT, width), np.float32)
        for k, i in enumerate(part):
            data[k, :, :, :lines[i].shape[2]] = lines[i]
        batches.append((data, len(part), width))
        order.extend(part)
    return batches, order


def _page_layout(seed: int, w: int, h: int, bands: int, line_h: int):
    """The ink rectangles of page(seed, ...), band by band: [(y0, y1, [(x0, x1), ...]), ...]."""
    rng = np.random.default_rng(seed + 2000)
    margin_y, margin_x = h * 150 // 3300, w * 150 // 2550
    pitch = (h - 2 * margin_y) / bands
    out = []
    for i in range(bands):
        y0 = int(margin_y + i * pitch)
        y1 = min(h, y0 + line_h)
        x = margin_x + int(rng.integers(0, 40))
        end = w - margin_x - int(rng.integers(0, 400))
        rects = []
        while x < end:
            rw = int(rng.integers(10, 61))
            rects.append((x, min(end, x + rw)))
            x += rw + int(rng.integers(4, 17)) + (int(rng.integers(20, 40)) if rng.random() < 0.15 else 0)
        out.append((y0, y1, rects))
    return out


def page_word_mask(seed: int = 1, w: int = 2550, h: int = 3300, bands: int = 36, line_h: int = 40,
                   grow_x: int = 8, grow_y: int = 3) -> np.ndarray:
    """The text mask a trained detector gives for page(seed, ...): bool [h, w], each ink
    rectangle grown by grow_x / grow_y (so the glyph gaps of a word close and the word gaps stay
    open), its top and bottom edges jittered by up to 2 px so the word outlines are ragged."""
    rng = np.random.default_rng(seed + 4000)
    m = np.zeros((h, w), bool)
    for y0, y1, rects in _page_layout(seed, w, h, bands, line_h):
        for x0, x1 in rects:
            t, b = y0 - grow_y + int(rng.integers(-2, 3)), y1 + grow_y + int(rng.integers(-2, 3))
            m[max(t, 0):min(b, h), max(x0 - grow_x, 0):min(x1 + grow_x, w)] = True
    return m


def pack_mask(m: np.ndarray) -> np.ndarray:
    """A bool mask [..., h, w] as the library's bit mask: uint32 [..., h, ceil(w / 32)], bit b of
    word j = pixel 32 j + b."""
    w = m.shape[-1]
    words = (w + 31) // 32
    pad = np.zeros(m.shape[:-1] + (words * 32,), bool)
    pad[..., :w] = m
    return np.packbits(pad.reshape(m.shape[:-1] + (words, 32)), axis=-1, bitorder="little").view("<u4")[..., 0].copy()


def page(seed: int = 1, w: int = 2550, h: int = 3300, bands: int = 36, line_h: int = 40,
         ink: int = 20) -> np.ndarray:
    """A US Letter page at 300 dpi as RGB u8 [h, w, 3]: white, with `bands` text lines of
    dark rectangles (width 10..60 px, gaps 4..16 px, a wider word gap now and then)."""
    img = np.full((h, w, 3), 255, np.uint8)
    for y0, y1, rects in _page_layout(seed, w, h, bands, line_h):
        for x0, x1 in rects:
            img[y0:y1, x0:x1] = ink
    return img


def page_db_candidates(seed: int, w: int, h: int, to_page, bands: int = 36, line_h: int = 40) -> np.ndarray:
    """DB box candidates of page(seed, ...) in detector-map coordinates, as `score` takes them
    ([cx, cy, up_x, up_y, width, height], src/ppdet.rs:63): every ink rectangle (a word piece)
    and every text line, axis-aligned, divided by the map-to-page factors `to_page`."""
    sx, sy = float(to_page[0]), float(to_page[1])
    out = []
    for y0, y1, rects in _page_layout(seed, w, h, bands, line_h):
        boxes = list(rects) + ([(rects[0][0], rects[-1][1])] if rects else [])
        for x0, x1 in boxes:
            out.append([(x0 + x1) / 2 / sx, (y0 + y1) / 2 / sy, 0.0, -1.0, (x1 - x0) / sx, (y1 - y0) / sy])
    return np.array(out, np.float32).reshape(-1, 6)


def page_line_boxes(seed: int = 1, w: int = 2550, h: int = 3300, bands: int = 36, line_h: int = 40,
                    relv: float = 0.1) -> np.ndarray:
    """The text lines of page(seed, ...) as recognition boxes [left, top, right, bottom] (f32):
    each band's ink extent, grown by relv x its height above and below, as the reference pads DB
    boxes (RELV 0.1, src/bin/ocr-bench.rs:538-556)."""
    boxes = []
    for y0, y1, rects in _page_layout(seed, w, h, bands, line_h):
        if not rects:
            continue
        pad = relv * (y1 - y0)
        boxes.append([rects[0][0], y0 - pad, rects[-1][1], y1 + pad])
    return np.array(boxes, np.float32)


def pages(seed: int = 1, n: int = 12, w: int = 2550, h: int = 3300) -> List[np.ndarray]:
    return [page(seed * 1000 + k, w, h) for k in range(n)]
