"""CPU oracle for the wgpu-ocr hot path -- TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py` may import this
module.  It is the checker, never the thing measured as the product.

Two layers:
  * ctypes wrappers around `oracle.c`, a C restatement of the reference's kernel arithmetic;
  * `run_onnx`, an interpreter of the (unfused) ONNX node list, standing in for the reference's
    stated oracle, "rten CPU execution of the same ONNX graph" (rten =0.26.0 is an un-vendored
    crates.io dependency and cannot run here).  Heavy float math goes to the C functions;
    broadcasting elementwise ops and reshapes use numpy in float32.

On top of those, the reference's pipeline entry points are restated:
  `detect_page`   - `Detector::detect_page`        src/gpu.rs:1393-1422
  `detect`        - `Detector::detect`             src/gpu.rs:1425-1430
  `recognize`     - `Recognizer::recognize`        src/gpu.rs:1510-1602 (per batch, as rten runs it)
  `det_input`     - `NdGraph::det_input`           src/nd.rs:1353-1369
  `ocrs_decode`   - greedy CTC of ocr-bench        src/bin/ocr-bench.rs:62-74
  `pp_decode`     - `Dictionary::decode`           src/ppocr.rs:23-33

Parity status: UNPINNED against the reference itself (no golden vectors exist in the reference,
and neither its Rust/wgpu path nor rten can run here); cross-checked against PyTorch CPU.
"""
from __future__ import annotations

import ctypes
import math
import os
import sys
from typing import Dict, List, Tuple

import numpy as np

from . import build as _build

_lib = None
_f = ctypes.POINTER(ctypes.c_float)
_u8 = ctypes.POINTER(ctypes.c_uint8)
_u32 = ctypes.POINTER(ctypes.c_uint32)
_i32 = ctypes.POINTER(ctypes.c_int32)
_I, _L, _F = ctypes.c_int, ctypes.c_long, ctypes.c_float


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        sig = {
            "oracle_conv2d": [_f, _I, _I, _I, _I, _f, _f, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _f, _f, _f],
            "oracle_convt": [_f, _I, _I, _I, _I, _f, _f, _I, _I, _I, _I, _I, _f],
            "oracle_pool": [_f, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _f],
            "oracle_grey_resize": [_u8, _I, _I, _I, _I, _f],
            "oracle_mask_up": [_f, _I, _I, _I, _I, _I, _F, _u32, _f],
            "oracle_det_prep": [_u8, _I, _I, _I, _I, _f],
            "oracle_resize_nearest": [_f, _I, _I, _I, _I, _I, _F, _F, _f],
            "oracle_gemm": [_f, _f, _f, _I, _I, _I, _I, _f],
            "oracle_gru": [_f, _f, _f, _i32, _I, _I, _I, _f],
            "oracle_avgpool_t": [_f, _I, _I, _I, _I, _I, _I, _I, _f],
            "oracle_layer_norm": [_f, _f, _f, _L, _I, _F, _f],
            "oracle_softmax": [_f, _L, _L, _f],
            "oracle_argmax": [_f, _L, _L, _u32, _f, _f, _f],
            "oracle_reduce_mean": [_f, _L, _L, _f],
            "oracle_bmm": [_f, _f, _L, _I, _I, _I, _f],
            "oracle_unary": [_f, _L, _I, _F, _F, _f],
            "oracle_set_threads": [_I],
            "oracle_threads": [],
            "oracle_erf": [_F],
            "oracle_act": [_F, _I],
            "oracle_pp_line": [_u8, _I, _I, _f, _f],
            "oracle_db_score": [_f, _I, _I, _f],
            "oracle_contours": [_u32, _I, _I, _i32, _I, _i32, _i32, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)],
            "oracle_word_rects": [_u32, _I, _I, _F, _F, _F, _f, _I],
            "oracle_db_boxes": [_f, _I, _I, _f, _F, _F, _F, _F, _f, _I],
            "oracle_text_lines": [_f, _I, _i32, _i32],
            "oracle_pad_line": [_f, _I, _F, _F],
            "oracle_ocrs_line": [_u8, _I, _I, _f, _I, _f, _i32],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_float if name in ("oracle_erf", "oracle_act", "oracle_db_score") else (
                ctypes.c_int if name in ("oracle_threads", "oracle_pp_line", "oracle_contours", "oracle_word_rects",
                                 "oracle_db_boxes", "oracle_text_lines", "oracle_ocrs_line")
                else None)
        _lib = L
    return _lib


def set_threads(n: int):
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return int(lib().oracle_threads())


def _p(a, t=_f):
    return None if a is None else a.ctypes.data_as(t)


def _c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# --------------------------------------------------------------------------------------------
# kernels
# --------------------------------------------------------------------------------------------
def conv2d(x, w, b=None, group=1, strides=(1, 1), pads=(0, 0, 0, 0), act=0, res=None, insc=None):
    """pads = (top, left, bottom, right)."""
    x, w = _c32(x), _c32(w)
    n, cin, h, wd = x.shape
    cout, _, kh, kw = w.shape
    pt, pl, pb, pr = pads
    oh = (h + pt + pb - kh) // strides[0] + 1
    ow = (wd + pl + pr - kw) // strides[1] + 1
    y = np.empty((n, cout, oh, ow), np.float32)
    b = None if b is None else _c32(b)
    res = None if res is None else _c32(res)
    insc = None if insc is None else _c32(insc)
    lib().oracle_conv2d(_p(x), n, cin, h, wd, _p(w), _p(b), cout, group, kh, kw, strides[0], strides[1],
                        pt, pl, pb, pr, act, _p(res), _p(insc), _p(y))
    return y


def convt(x, w, b=None, stride=2, act=0):
    x, w = _c32(x), _c32(w)
    n, cin, h, wd = x.shape
    _, cout, kh, kw = w.shape
    y = np.empty((n, cout, (h - 1) * stride + kh, (wd - 1) * stride + kw), np.float32)
    b = None if b is None else _c32(b)
    lib().oracle_convt(_p(x), n, cin, h, wd, _p(w), _p(b), cout, kh, kw, stride, act, _p(y))
    return y


def pool(x, kh, kw, sh, sw, pads=(0, 0, 0, 0), avg=False):
    x = _c32(x)
    n, c, h, w = x.shape
    pt, pl, pb, pr = pads
    oh = (h + pt + pb - kh) // sh + 1
    ow = (w + pl + pr - kw) // sw + 1
    y = np.empty((n, c, oh, ow), np.float32)
    lib().oracle_pool(_p(x), n * c, h, w, oh, ow, kh, kw, sh, sw, pt, pl, int(avg), _p(y))
    return y


def contours(bits: np.ndarray, w: int, h: int):
    """find_contours(mask, External) of a bit mask (uint32 [h, ceil(w / 32)]): a list of int32
    [n, 2] (x, y) point arrays in raster order of their start pixels."""
    bits = np.ascontiguousarray(bits, np.uint32)
    np_ = ctypes.c_int64()
    nc = lib().oracle_contours(_p(bits, _u32), w, h, None, 0, None, None, 0, ctypes.byref(np_))
    lens = np.zeros(max(nc, 1), np.int32)
    xs = np.zeros(max(np_.value, 1), np.int32)
    ys = np.zeros(max(np_.value, 1), np.int32)
    lib().oracle_contours(_p(bits, _u32), w, h, _p(lens, _i32), nc, _p(xs, _i32), _p(ys, _i32), np_.value,
                          ctypes.byref(np_))
    out, o = [], 0
    for n in lens[:nc]:
        out.append(np.stack([xs[o:o + n], ys[o:o + n]], 1))
        o += n
    return out


def word_rects(bits: np.ndarray, w: int, h: int, expand: float = 3.0, expand_x: float = 0.0,
               min_area: float = 100.0) -> np.ndarray:
    """word_rects (src/bin/ocr-bench.rs:38-60) of a bit mask: float32 [n, 6] rectangles
    [cx, cy, up_x, up_y, width, height] in contour order."""
    bits = np.ascontiguousarray(bits, np.uint32)
    n = lib().oracle_word_rects(_p(bits, _u32), w, h, expand, expand_x, min_area, None, 0)
    out = np.zeros((max(n, 1), 6), np.float32)
    lib().oracle_word_rects(_p(bits, _u32), w, h, expand, expand_x, min_area, _p(out), n)
    return out[:n]


def db_boxes(prob: np.ndarray, to_page, thresh: float = 0.2, box_thresh: float = 0.45, unclip_ratio: float = 1.4,
             min_size: float = 3.0) -> np.ndarray:
    """ppdet::boxes (src/ppdet.rs:87-132) of a probability map [h, w]: float32 [n, 6] boxes
    [cx, cy, up_x, up_y, width, height] in page coordinates, in reading order (defaults:
    ppdet::Db::default())."""
    prob = np.ascontiguousarray(prob, np.float32)
    h, w = prob.shape
    tp = np.ascontiguousarray(to_page, np.float32)
    n = lib().oracle_db_boxes(_p(prob), w, h, _p(tp), thresh, box_thresh, unclip_ratio, min_size, None, 0)
    out = np.zeros((max(n, 1), 6), np.float32)
    lib().oracle_db_boxes(_p(prob), w, h, _p(tp), thresh, box_thresh, unclip_ratio, min_size, _p(out), n)
    return out[:n]


def db_scores(prob: np.ndarray, rects) -> np.ndarray:
    """`score` of src/ppdet.rs:63-83 for each box [cx, cy, up_x, up_y, width, height] of a
    probability map [h, w]."""
    prob = np.ascontiguousarray(prob, np.float32)
    h, w = prob.shape
    out = []
    for r in np.asarray(rects, np.float32).reshape(-1, 6):
        rr = np.ascontiguousarray(r)
        out.append(lib().oracle_db_score(_p(prob), w, h, _p(rr)))
    return np.array(out, np.float32)


def pp_line(rgb: np.ndarray, rect) -> np.ndarray:
    """One PP-OCR recognition line, [3, 48, out_w] in [-1, 1] (src/ppocr.rs:39-62; the Triangle
    resize of image =0.25.10 restated in oracle.c)."""
    rgb = np.ascontiguousarray(rgb, np.uint8)
    h, w = rgb.shape[:2]
    r = np.ascontiguousarray(rect, np.float32)
    ow = lib().oracle_pp_line(_p(rgb, _u8), w, h, _p(r), None)
    out = np.empty((3, 48, ow), np.float32)
    lib().oracle_pp_line(_p(rgb, _u8), w, h, _p(r), _p(out))
    return out


def pp_line_rects(boxes, relv: float = 0.1) -> np.ndarray:
    """The line rectangles [left, top, right, bottom] of DB boxes as the page pipeline cuts them
    (src/bin/ocr-bench.rs:534-558 and 312-321: each box its own line, grown by relv x its height
    across the text, then its bounding rectangle), in f32."""
    f = np.float32
    out = []
    for cx, cy, ux, uy, bw, bh in np.asarray(boxes, np.float32).reshape(-1, 6):
        upright = abs(uy) >= abs(ux)
        across = f(relv) * (bh if upright else bw)
        rw = bw if upright else f(bw + f(2) * across)
        rh = f(bh + f(2) * across) if upright else bh
        hw, hh = rw / f(2), rh / f(2)
        xs = [cx + f(sa) * hh * ux + f(sb) * hw * -uy for sa in (-1, 1) for sb in (-1, 1)]
        ys = [cy + f(sa) * hh * uy + f(sb) * hw * ux for sa in (-1, 1) for sb in (-1, 1)]
        out.append([min(xs), min(ys), max(xs), max(ys)])
    return np.array(out, np.float32).reshape(-1, 4)


def pp_batches(rgb: np.ndarray, rects, per: int = 16):
    """PP-OCR line batches as src/bin/ocr-bench.rs:312-345 forms them (PPGROUP = 0): lines sorted
    by width (stable), cut into batches of `per`, each [n, 3, 48, width] with width the widest
    line rounded up to a multiple of 8, zero-padded on the right.  Returns (batches as
    (data, n, width), order: the line index of each batch slot)."""
    lines = [pp_line(rgb, r) for r in rects]
    idx = sorted(range(len(lines)), key=lambda i: lines[i].shape[2])
    batches, order = [], []
    for k in range(0, len(idx), per):
        part = idx[k:k + per]
        width = -(-max(lines[i].shape[2] for i in part) // 8) * 8
        data = np.zeros((len(part), 3, 48, width), np.float32)
        for j, i in enumerate(part):
            data[j, :, :, :lines[i].shape[2]] = lines[i]
        batches.append((data, len(part), width))
        order.extend(part)
    return batches, order


def text_lines(words) -> List[List[int]]:
    """ocrs' find_text_lines as restated in oracle.c (parity unpinned): the word indices of each
    line, lines in reading order, words left to right."""
    r = np.ascontiguousarray(np.asarray(words, np.float32).reshape(-1, 6))
    n = len(r)
    order = np.zeros(max(n, 1), np.int32)
    lens = np.zeros(max(n, 1), np.int32)
    nl = lib().oracle_text_lines(_p(r), n, _p(order, _i32), _p(lens, _i32))
    out, o = [], 0
    for k in range(nl):
        out.append(order[o:o + lens[k]].tolist())
        o += int(lens[k])
    return out


def pad_line(words, relv: float = 0.15, relend: float = 0.1) -> np.ndarray:
    """The words of one line padded as src/bin/ocr-bench.rs:534-558 pads them."""
    r = np.array(np.asarray(words, np.float32).reshape(-1, 6), np.float32, copy=True)
    lib().oracle_pad_line(_p(r), len(r), relv, relend)
    return r


def ocrs_line(rgb: np.ndarray, words):
    """The 64-row ocrs line image [64, W] of one (padded) line, and its crop [l, t, w, h]."""
    rgb = np.ascontiguousarray(rgb, np.uint8)
    h, w = rgb.shape[:2]
    r = np.ascontiguousarray(np.asarray(words, np.float32).reshape(-1, 6))
    crop = np.zeros(4, np.int32)
    W = lib().oracle_ocrs_line(_p(rgb, _u8), w, h, _p(r), len(r), None, _p(crop, _i32))
    out = np.empty((64, W), np.float32)
    lib().oracle_ocrs_line(_p(rgb, _u8), w, h, _p(r), len(r), _p(out), None)
    return out, crop


def ocrs_page_lines(bits: np.ndarray, w: int, h: int, relv: float = 0.15, relend: float = 0.1):
    """The host half of the ocrs page pipeline on a page mask: word rectangles (expand 3, min
    area 100), text lines, padding.  Returns the padded words of each line (float32 [k, 6])."""
    words = word_rects(bits, w, h)
    return [pad_line(words[idx], relv, relend) for idx in text_lines(words)]


def ocrs_line_batches(rgb: np.ndarray, lines, bucket: int = 50, per: int = 20):
    """line_batches (src/bin/ocr-bench.rs:365-408): each line's image, grouped by width rounded
    up to `bucket` (ascending), `per` lines a batch in line order, padded with -0.5.  Returns
    (batches as (data [n, 1, 64, width], n, width), order: line of each slot, widths: each slot's
    image width)."""
    imgs = [ocrs_line(rgb, l)[0] for l in lines]
    groups = {}
    for i, im in enumerate(imgs):
        groups.setdefault(-(-im.shape[1] // bucket) * bucket, []).append(i)
    batches, order, widths = [], [], []
    for width in sorted(groups):
        mem = groups[width]
        for k in range(0, len(mem), per):
            part = mem[k:k + per]
            data = np.full((len(part), 1, 64, width), -0.5, np.float32)
            for j, i in enumerate(part):
                data[j, 0, :, :imgs[i].shape[1]] = imgs[i]
                order.append(i)
                widths.append(imgs[i].shape[1])
            batches.append((data, len(part), width))
    return batches, order, widths


def grey_resize(rgb: np.ndarray, oh: int = 800, ow: int = 600) -> np.ndarray:
    h, w, _ = rgb.shape
    rgb = np.ascontiguousarray(rgb, np.uint8)
    y = np.empty((oh, ow), np.float32)
    lib().oracle_grey_resize(_p(rgb, _u8), w, h, ow, oh, _p(y))
    return y


def mask_up(m: np.ndarray, vw: int, vh: int, w: int, h: int, thr: float):
    """m: [mh, stride] model map; returns (bits [h, ceil(w/32)] u32, prob [h, w] f32)."""
    m = _c32(m)
    stride = m.shape[1]
    words = (w + 31) // 32
    bits = np.empty((h, words), np.uint32)
    prob = np.empty((h, w), np.float32)
    lib().oracle_mask_up(_p(m), stride, vw, vh, w, h, thr, _p(bits, _u32), _p(prob))
    return bits, prob


def det_prep(rgb: np.ndarray, ow: int, oh: int) -> np.ndarray:
    h, w, _ = rgb.shape
    rgb = np.ascontiguousarray(rgb, np.uint8)
    y = np.empty((1, 3, oh, ow), np.float32)
    lib().oracle_det_prep(_p(rgb, _u8), w, h, ow, oh, _p(y))
    return y


def resize_nearest(x, sy, sx):
    x = _c32(x)
    n, c, h, w = x.shape
    oh, ow = int(math.floor(h * sy)), int(math.floor(w * sx))
    y = np.empty((n, c, oh, ow), np.float32)
    lib().oracle_resize_nearest(_p(x), n * c, h, w, oh, ow, sy, sx, _p(y))
    return y


def gemm(x, wt, b=None, act=0):
    x, wt = _c32(x), _c32(wt)
    m, i = x.shape
    k = wt.shape[1]
    y = np.empty((m, k), np.float32)
    b = None if b is None else _c32(b)
    lib().oracle_gemm(_p(x), _p(wt), _p(b), m, k, i, act, _p(y))
    return y


def gru(g, r, rb, lens, hid=256):
    """g [tmax, ntot, 2*3*hid]; r [2, 3*hid, hid]; rb [2, 3*hid]; returns y [tmax, ntot, 2*hid]
    (NaN where t >= len: the reference never writes those rows)."""
    g, r, rb = _c32(g), _c32(r), _c32(rb)
    tmax, ntot = g.shape[0], g.shape[1]
    lens = np.ascontiguousarray(lens, np.int32)
    y = np.full((tmax, ntot, 2 * hid), np.nan, np.float32)
    lib().oracle_gru(_p(g), _p(r), _p(rb), _p(lens, _i32), tmax, ntot, hid, _p(y))
    return y


def layer_norm(x, gamma, beta, eps):
    x = _c32(x)
    n = x.shape[-1]
    y = np.empty_like(x)
    lib().oracle_layer_norm(_p(x), _p(_c32(gamma)), _p(_c32(beta)), x.size // n, n, eps, _p(y))
    return y


def softmax(x, axis=-1):
    x = np.moveaxis(_c32(x), axis, -1).copy() if axis not in (-1, x.ndim - 1) else _c32(x)
    n = x.shape[-1]
    y = np.empty_like(x)
    lib().oracle_softmax(_p(x), x.size // n, n, _p(y))
    return y


def argmax(x):
    """Row arg-max over the last axis (ties -> lowest index) with top-1, top-2 and logsumexp."""
    x = _c32(x)
    n = x.shape[-1]
    rows = x.size // n
    best = np.empty(rows, np.uint32)
    t1, t2, lse = (np.empty(rows, np.float32) for _ in range(3))
    lib().oracle_argmax(_p(x), rows, n, _p(best, _u32), _p(t1), _p(t2), _p(lse))
    shp = x.shape[:-1]
    return best.reshape(shp), t1.reshape(shp), t2.reshape(shp), lse.reshape(shp)


def reduce_mean_trailing(x, naxes):
    x = _c32(x)
    inner = int(np.prod(x.shape[x.ndim - naxes:]))
    outer = x.size // max(inner, 1)
    y = np.empty(outer, np.float32)
    lib().oracle_reduce_mean(_p(x), outer, inner, _p(y))
    return y


def bmm(a, c):
    a, c = _c32(a), _c32(c)
    bshape = a.shape[:-2]
    batch = int(np.prod(bshape)) if bshape else 1
    m, k = a.shape[-2:]
    n = c.shape[-1]
    y = np.empty(bshape + (m, n), np.float32)
    lib().oracle_bmm(_p(a), _p(c), batch, m, k, n, _p(y))
    return y


def unary(x, op, alpha=0.2, beta=0.5):
    x = _c32(x)
    y = np.empty_like(x)
    lib().oracle_unary(_p(x), x.size, op, alpha, beta, _p(y))
    return y


# --------------------------------------------------------------------------------------------
# ONNX interpreter (rten stand-in)
# --------------------------------------------------------------------------------------------
class _Int:
    """An integer tensor kept on the host (shapes and indices), as in src/nd.rs:448-453."""

    def __init__(self, v, shape=None):
        self.v = np.asarray(v, np.int64).reshape(-1)
        self.shape = list(shape) if shape is not None else ([self.v.size] if self.v.size != 1 else [1])


def _pads(node, h, w, kh, kw, sh, sw):
    """Leading/trailing padding; SAME_UPPER puts the odd one at the end (src/nd.rs:1270-1278)."""
    if node.string("auto_pad") == "SAME_UPPER":
        oh, ow = -(-h // sh), -(-w // sw)
        th = max((oh - 1) * sh + kh - h, 0)
        tw = max((ow - 1) * sw + kw - w, 0)
        return th // 2, tw // 2, th - th // 2, tw - tw // 2
    p = node.ints("pads") or [0, 0, 0, 0]
    return p[0], p[1], p[2], p[3]


def _axis(a, r):
    return a + r if a < 0 else a


def run_onnx(model, x: np.ndarray, stop_before_softmax: bool = False, trace=None, values=None) -> np.ndarray:
    """Run `model` (a `wocr.model.Model`) on `x` with plain ONNX semantics, node by node.
    `values` (a dict) receives every computed value by name."""
    vals: Dict[str, object] = {model.input: _c32(x)}
    nodes = list(model.nodes)
    out_name = model.output
    if stop_before_softmax and nodes and nodes[-1].op == "Softmax" and nodes[-1].outputs[0] == out_name:
        out_name = nodes[-1].inputs[0]
        nodes = nodes[:-1]

    def get(name):
        if name in vals:
            return vals[name]
        if name in model.weights:
            return model.weights[name]
        if name in model.ints:
            return _Int(model.ints[name])
        raise KeyError(f"missing value {name}")

    def flt(name):
        v = get(name)
        if isinstance(v, _Int):
            raise TypeError(f"{name} is an integer tensor")
        return v

    for nd in nodes:
        op = nd.op
        a = lambda k: get(nd.inputs[k])  # noqa: E731
        if op == "Identity":
            y = a(0)
        elif op == "Conv":
            xin, w = flt(nd.inputs[0]), flt(nd.inputs[1])
            b = flt(nd.inputs[2]) if len(nd.inputs) > 2 and nd.inputs[2] else None
            st = nd.ints("strides") or [1, 1]
            kh, kw = w.shape[2], w.shape[3]
            pads = _pads(nd, xin.shape[2], xin.shape[3], kh, kw, st[0], st[1])
            y = conv2d(xin, w, b, group=nd.int("group") or 1, strides=st, pads=pads)
        elif op == "ConvTranspose":
            xin, w = flt(nd.inputs[0]), flt(nd.inputs[1])
            b = flt(nd.inputs[2]) if len(nd.inputs) > 2 and nd.inputs[2] else None
            y = convt(xin, w, b, stride=(nd.ints("strides") or [1, 1])[0])
        elif op in ("MaxPool", "AveragePool"):
            xin = flt(nd.inputs[0])
            k = nd.ints("kernel_shape")
            st = nd.ints("strides") or [1, 1]
            pads = _pads(nd, xin.shape[2], xin.shape[3], k[0], k[1], st[0], st[1])
            y = pool(xin, k[0], k[1], st[0], st[1], pads, avg=(op == "AveragePool"))
        elif op == "GlobalAveragePool":
            xin = flt(nd.inputs[0])
            y = reduce_mean_trailing(xin, xin.ndim - 2).reshape(xin.shape[:2] + (1,) * (xin.ndim - 2))
        elif op == "BatchNormalization":
            xin = flt(nd.inputs[0])
            g, bb, m, v = (flt(nd.inputs[i]) for i in range(1, 5))
            eps = nd.attr_f32("epsilon")
            eps = 1e-5 if eps is None else eps
            s = (g / np.sqrt(v + np.float32(eps))).astype(np.float32)
            sh = (bb - m * s).astype(np.float32)
            shp = (1, -1) + (1,) * (xin.ndim - 2)
            y = (xin * s.reshape(shp) + sh.reshape(shp)).astype(np.float32)
        elif op in ("Relu", "Sigmoid", "HardSigmoid", "Erf", "Sqrt"):
            code = {"Relu": 1, "Sigmoid": 2, "HardSigmoid": 3, "Erf": 4, "Sqrt": 5}[op]
            al = nd.attr_f32("alpha")
            be = nd.attr_f32("beta")
            y = unary(flt(nd.inputs[0]), code, 0.2 if al is None else al, 0.5 if be is None else be)
        elif op in ("Add", "Sub", "Mul", "Div", "Pow"):
            p, q = a(0), a(1)
            if isinstance(p, _Int) and isinstance(q, _Int):
                f = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply}.get(op)
                if op == "Div":
                    r = np.where(q.v == 0, 0, p.v // np.where(q.v == 0, 1, q.v))
                elif f is None:
                    r = p.v
                else:
                    r = f(p.v, q.v)
                y = _Int(r, p.shape)
            else:
                p, q = np.asarray(p, np.float32), np.asarray(q, np.float32)
                if op == "Add":
                    y = p + q
                elif op == "Sub":
                    y = p - q
                elif op == "Mul":
                    y = p * q
                elif op == "Div":
                    y = p / q
                else:
                    if q.size == 1 and float(q.reshape(-1)[0]) == 2.0:
                        y = p * p
                    elif q.size == 1 and float(q.reshape(-1)[0]) == 0.5:
                        y = np.sqrt(p)
                    else:
                        y = np.power(p, q)
                y = np.ascontiguousarray(y, np.float32)
        elif op == "ReduceMean":
            xin = flt(nd.inputs[0])
            r = xin.ndim
            axes = sorted(_axis(v, r) for v in (nd.ints("axes") or list(range(r))))
            if axes != list(range(r - len(axes), r)):
                raise ValueError("ReduceMean over non-trailing axes")
            keep = (nd.int("keepdims") if nd.int("keepdims") is not None else 1) == 1
            y = reduce_mean_trailing(xin, len(axes))
            shp = [s if d not in axes else 1 for d, s in enumerate(xin.shape) if (d not in axes or keep)]
            y = y.reshape(shp)
        elif op == "Softmax":
            xin = flt(nd.inputs[0])
            ax = _axis(nd.int("axis") if nd.int("axis") is not None else -1, xin.ndim)
            inner = int(np.prod(xin.shape[ax:]))
            y = softmax(xin.reshape(-1, inner)).reshape(xin.shape)
        elif op == "MatMul":
            p, q = flt(nd.inputs[0]), flt(nd.inputs[1])
            if nd.inputs[1] in model.weights and q.ndim == 2:
                lead = p.shape[:-1]
                y = gemm(p.reshape(-1, p.shape[-1]), q).reshape(lead + (q.shape[1],))
            else:
                y = bmm(p, q)
        elif op == "Transpose":
            xin = flt(nd.inputs[0])
            perm = nd.ints("perm") or list(range(xin.ndim))[::-1]
            y = np.ascontiguousarray(np.transpose(xin, perm))
        elif op == "Reshape":
            xin = flt(nd.inputs[0])
            want = list(a(1).v)
            shape = [xin.shape[d] if s == 0 else max(int(s), 1) for d, s in enumerate(want)]
            if -1 in want:
                p = want.index(-1)
                known = int(np.prod([s for d, s in enumerate(shape) if d != p]))
                shape[p] = xin.size // max(known, 1)
            y = xin.reshape(shape)
        elif op in ("Squeeze", "Unsqueeze"):
            axes = nd.ints("axes") if nd.ints("axes") is not None else list(a(1).v)
            v = a(0)
            if isinstance(v, _Int):
                y = _Int(v.v, [d for d in v.shape if d != 1] if op == "Squeeze" else [v.v.size])
            elif op == "Squeeze":
                y = np.squeeze(v, tuple(_axis(x_, v.ndim) for x_ in axes))
            else:
                r = v.ndim + len(axes)
                y = np.expand_dims(v, tuple(_axis(x_, r) for x_ in axes))
        elif op == "Slice":
            data = a(0)
            starts, ends = list(a(1).v), list(a(2).v)
            axes = list(a(3).v) if len(nd.inputs) > 3 and nd.inputs[3] else list(range(len(starts)))
            if len(nd.inputs) > 4 and nd.inputs[4] and any(s != 1 for s in a(4).v):
                raise ValueError("Slice with steps")
            shape = data.shape if not isinstance(data, _Int) else data.shape
            sl = [slice(None)] * len(shape)
            for st, en, ax in zip(starts, ends, axes):
                ax = _axis(int(ax), len(shape))
                dim = shape[ax]
                cl = lambda v: min(max(v + dim if v < 0 else v, 0), dim)  # noqa: E731
                sl[ax] = slice(cl(int(st)), cl(int(en)))
            if isinstance(data, _Int):
                y = _Int(data.v[sl[0]])
            else:
                y = np.ascontiguousarray(data[tuple(sl)])
        elif op == "Concat":
            parts = [a(k) for k in range(len(nd.inputs))]
            if all(isinstance(p, _Int) for p in parts):
                y = _Int(np.concatenate([p.v for p in parts]))
            else:
                y = np.concatenate(parts, axis=nd.int("axis") or 0).astype(np.float32)
        elif op == "Shape":
            v = a(0)
            y = _Int(list(v.shape))
        elif op == "Gather":
            d, idx = a(0), a(1)
            vv = [d.v[i + d.v.size if i < 0 else i] for i in idx.v]
            y = _Int(vv, [] if len(vv) == 1 else [len(vv)])
        elif op == "Cast":
            y = a(0)
        elif op == "Pad":
            y = flt(nd.inputs[0])
            pads = get(nd.inputs[1]) if len(nd.inputs) > 1 else None
            pv = pads.v if isinstance(pads, _Int) else (np.asarray(pads).reshape(-1) if pads is not None else [])
            if any(int(v) != 0 for v in pv):
                raise ValueError("non-zero Pad")
        elif op == "Resize":
            xin = flt(nd.inputs[0])
            sc = model.weights[nd.inputs[2]].reshape(-1)
            y = resize_nearest(xin, float(sc[2]), float(sc[3]))
        elif op == "GRU":
            y = _onnx_gru(flt(nd.inputs[0]), flt(nd.inputs[1]), flt(nd.inputs[2]), flt(nd.inputs[3]),
                          nd.int("hidden_size"))
        else:
            raise ValueError(f"unsupported op {op}")
        vals[nd.outputs[0]] = y
        if values is not None:
            values[nd.outputs[0]] = y
        if trace is not None:
            trace.append((nd.op, nd.outputs[0], getattr(y, "shape", None)))
    out = vals[out_name]
    return out


def _onnx_gru(X, W, R, B, hid):
    """ONNX GRU, bidirectional, linear_before_reset = 1, no sequence_lens: Y [T, 2, n, hid]."""
    T, n, inp = X.shape
    G = 3 * hid
    g = np.empty((T, n, 2, G), np.float32)
    for d in range(2):
        g[:, :, d, :] = gemm(X.reshape(-1, inp), np.ascontiguousarray(W[d].T), B[d, :G]).reshape(T, n, G)
    y = gru(g.reshape(T, n, 2 * G), R, B[:, G:], np.full(n, T, np.int32), hid)
    return np.ascontiguousarray(y.reshape(T, n, 2, hid).transpose(0, 2, 1, 3))


# --------------------------------------------------------------------------------------------
# pipeline entry points of the reference, restated
# --------------------------------------------------------------------------------------------
def detect_valid(w: int, h: int, mh: int = 800, mw: int = 600):
    """Padded size and the valid part of the model map (src/gpu.rs:1394-1416)."""
    ph, pw = max(h, mh), max(w, mw)
    vh = mh - (ph - h) * mh // ph
    vw = mw - (pw - w) * mw // pw
    return ph, pw, vh, vw


def detect_page(model, rgb: np.ndarray, thr: float):
    """Detector::detect_page: returns (bits [h, ceil(w/32)], page-level prob [h, w], model map)."""
    h, w, _ = rgb.shape
    inp = grey_resize(rgb, 800, 600)
    m = run_onnx(model, inp.reshape(1, 1, 800, 600))
    _, _, vh, vw = detect_valid(w, h)
    bits, prob = mask_up(m.reshape(800, 600), vw, vh, w, h, thr)
    return bits, prob, m


def detect(model, inp: np.ndarray) -> np.ndarray:
    """Detector::detect: the probability map of a [1, 1, h, w] input."""
    return run_onnx(model, inp)


def recognize(model, batches):
    """Recognizer::recognize, each batch run through the whole ONNX graph as rten runs it.
    Returns (logits [tmax, ntot, classes] (NaN where t >= len), tmax, lens)."""
    outs = [run_onnx(model, data) for data, _, _ in batches]   # [T_b, n_b, classes]
    tmax = max(o.shape[0] for o in outs)
    ntot = sum(o.shape[1] for o in outs)
    classes = outs[0].shape[2]
    logits = np.full((tmax, ntot, classes), np.nan, np.float32)
    lens = []
    off = 0
    for o in outs:
        t, nb, _ = o.shape
        logits[:t, off:off + nb] = o
        lens += [t] * nb
        off += nb
    return logits, tmax, lens


def det_input_size(w: int, h: int, max_side: int):
    """Sizes chosen by det_input (src/nd.rs:1354-1357, src/ppdet.rs:29-33)."""
    ratio = max_side / max(w, h) if max(w, h) > max_side else 1.0
    rnd = lambda v: max(int(round(v / 32.0)) * 32, 32)  # noqa: E731
    return rnd(w * np.float32(ratio)), rnd(h * np.float32(ratio))


def det_input(rgb: np.ndarray, max_side: int):
    """NdGraph::det_input: [1, 3, oh, ow] and the factors back to the page."""
    h, w, _ = rgb.shape
    ow, oh = det_input_size(w, h, max_side)
    return det_prep(rgb, ow, oh), (w / ow, h / oh)


def ocrs_best(row: np.ndarray) -> int:
    """Rust `max_by(total_cmp)` over a row: the LAST index among equal maxima."""
    m = np.max(row)
    return int(np.nonzero(row == m)[0][-1])


def ocrs_decode(logits, line: int, steps: int, width: int, alphabet: str) -> str:
    """Greedy CTC of src/bin/ocr-bench.rs:62-74 (drops characters starting at t*4 >= width)."""
    s, prev = [], 0
    for t in range(steps):
        best = ocrs_best(logits[t, line])
        if best != 0 and best != prev and t * 4 < width:
            s.append(alphabet[best - 1])
        prev = best
    return "".join(s)


def pp_decode(best, chars: List[str]) -> str:
    """Dictionary::decode (src/ppocr.rs:23-33): repeats merged, blanks dropped."""
    out, prev = [], 0
    for c in best:
        c = int(c)
        if c != 0 and c != prev:
            out.append(chars[c] if c < len(chars) else "")
        prev = c
    return "".join(out)
