"""The reference crate's public API for the hot path, over the C ABI.

  Gpu         - src/gpu.rs:825-1056   (`Gpu::new(lines)`, submit_wait, pool)
  Detector    - src/gpu.rs:1380-1431  (`new`, `detect_page`, `detect`)
  Recognizer  - src/gpu.rs:1433-1603  (`new`, `recognize`)
  NdGraph     - src/nd.rs:428-1394    (`new`, `run`, `argmax`, `det_input`)

Errors are raised as `WocrError` (the reference returns `Err(String)` from the same calls).
All work runs in hand-written sm_100a kernels of libwocr.so; nothing here computes on the CPU
except the greedy CTC decode, which the reference also runs on the host.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import _lib as L
from .model import Model


class Gpu:
    """`Gpu::new(lines)` (src/gpu.rs:850): one CUDA device, one stream, a pooled allocator."""

    def __init__(self, lines: int = 8, device: int = 0):
        h = ctypes.c_void_p()
        L.check(L.lib().wocr_ctx_create(int(device), int(lines), ctypes.byref(h)))
        self.h = h
        self.device = device
        self.lines = lines

    @property
    def adapter(self) -> str:
        buf = ctypes.create_string_buffer(256)
        L.check(L.lib().wocr_ctx_describe(self.h, buf, 256))
        return buf.value.decode()

    @property
    def stream(self) -> int:
        """The cudaStream_t all work of this device context runs on."""
        return int(L.lib().wocr_ctx_stream(self.h) or 0)

    def submit_wait(self, timeout_ms: int = 0):
        """Wait for all queued work (src/gpu.rs:1005-1008), optionally bounded."""
        L.check(L.lib().wocr_ctx_sync(self.h, int(timeout_ms)))

    def pool_bytes(self) -> int:
        return int(L.lib().wocr_ctx_pool_bytes(self.h))

    def launches(self) -> int:
        return int(L.lib().wocr_ctx_launches(self.h))

    def pp_lines(self, d_rgb: int, w: int, h: int, rects, per_batch: int = 16, d_out: int = 0, cap: int = 0):
        """PP-OCR recognition line batches cut from a device page (`wocr_pp_lines`): returns
        (order, [(n, width)] per batch, total floats).  With d_out (a device float buffer of `cap`
        floats) the batches are written there, one after another, [n, 3, 48, width] each."""
        r = np.ascontiguousarray(rects, np.float32).reshape(-1, 4)
        n = r.shape[0]
        order = np.zeros(max(n, 1), np.int32)
        bn = np.zeros(max(n, 1), np.int32)
        bw = np.zeros(max(n, 1), np.int32)
        nb, tot = ctypes.c_int32(), ctypes.c_int64()
        L.check(L.lib().wocr_pp_lines(self.h, ctypes.c_void_p(d_rgb), int(w), int(h), L.ptr(r), n, int(per_batch),
                                      ctypes.c_void_p(d_out or None), int(cap), L.ptr(order), L.ptr(bn), L.ptr(bw),
                                      ctypes.byref(nb), ctypes.byref(tot)))
        return order[:n].tolist(), [(int(bn[i]), int(bw[i])) for i in range(nb.value)], tot.value

    def ocrs_lines(self, d_rgb: int, w: int, h: int, lines, d_out: int = 0, cap: int = 0):
        """ocrs line images cut from a device page (`wocr_ocrs_lines`): `lines` = the padded words
        of each line (float32 [k, 6] each).  Returns (slots: the line of each batch slot, widths:
        each slot's image width, [(n, width)] per batch, total floats); with d_out (a device float
        buffer of `cap` floats) the batches [n, 1, 64, width] are written there one after another."""
        ws = [np.asarray(l, np.float32).reshape(-1, 6) for l in lines]
        words = np.ascontiguousarray(np.concatenate(ws) if ws else np.zeros((0, 6), np.float32))
        lens = np.array([len(x) for x in ws] or [0], np.int32)
        n = len(ws)
        slots = np.zeros(max(n, 1), np.int32)
        widths = np.zeros(max(n, 1), np.int32)
        bn = np.zeros(max(n, 1), np.int32)
        bw = np.zeros(max(n, 1), np.int32)
        nb, tot = ctypes.c_int32(), ctypes.c_int64()
        L.check(L.lib().wocr_ocrs_lines(self.h, ctypes.c_void_p(d_rgb or None), int(w), int(h), L.ptr(words),
                                        L.ptr(lens), n, ctypes.c_void_p(d_out or None), int(cap), L.ptr(slots),
                                        L.ptr(widths), L.ptr(bn), L.ptr(bw), ctypes.byref(nb), ctypes.byref(tot)))
        return (slots[:n].tolist(), widths[:n].tolist(), [(int(bn[i]), int(bw[i])) for i in range(nb.value)],
                tot.value)

    def word_rects(self, mask, w: int, h: int, expand: float = 3.0, expand_x: float = 0.0,
                   min_area: float = 100.0, d_mask: int = 0, n: int = 0):
        """word_rects (src/bin/ocr-bench.rs:38-60) of bit masks on the device (`wocr_word_rects`):
        `mask` uint32 [n, h, ceil(w / 32)] (or [h, words] for one page) in host memory, or
        d_mask, a device pointer to n such pages.  Returns a list per page of float32 [k, 6]
        rectangles [cx, cy, up_x, up_y, width, height]."""
        if d_mask:
            src, npg = ctypes.c_void_p(d_mask), int(n)
        else:
            m = np.ascontiguousarray(mask, np.uint32)
            npg = 1 if m.ndim == 2 else m.shape[0]
            src = L.ptr(m)
        counts = np.zeros(max(npg, 1), np.int32)
        out = np.zeros((4096 * max(npg, 1), 6), np.float32)
        for _ in range(2):  # again only when the first guess of the capacity was short (status 8)
            st = L.lib().wocr_word_rects(self.h, src, npg, int(w), int(h), int(bool(d_mask)), expand, expand_x,
                                         min_area, L.ptr(out), out.shape[0], L.ptr(counts))
            if st == 8 and counts[:npg].sum() > out.shape[0]:
                out = np.zeros((int(counts[:npg].sum()), 6), np.float32)
                continue
            L.check(st)
            break
        ends = np.cumsum(counts[:npg])
        return [out[e - k:e] for e, k in zip(ends, counts[:npg])]

    def db_boxes(self, prob, to_page, thresh: float = 0.2, box_thresh: float = 0.45, unclip_ratio: float = 1.4,
                 min_size: float = 3.0, d_prob: int = 0, w: int = 0, h: int = 0) -> np.ndarray:
        """ppdet::boxes (src/ppdet.rs:87-132) of a probability map (`wocr_db_boxes`): `prob`
        float32 [h, w] in host memory, or d_prob, a device pointer to a w x h map."""
        if d_prob:
            src, dev = ctypes.c_void_p(d_prob), 1
        else:
            prob = np.ascontiguousarray(prob, np.float32)
            h, w = prob.shape
            src, dev = L.ptr(prob), 0
        tp = np.ascontiguousarray(to_page, np.float32)
        n = ctypes.c_int32()
        out = np.zeros((1024, 6), np.float32)
        for _ in range(2):  # again only when the first guess of the capacity was short (status 8)
            st = L.lib().wocr_db_boxes(self.h, src, int(w), int(h), dev, L.ptr(tp), thresh, box_thresh, unclip_ratio,
                                       min_size, L.ptr(out), out.shape[0], ctypes.byref(n))
            if st == 8 and n.value > out.shape[0]:
                out = np.zeros((n.value, 6), np.float32)
                continue
            L.check(st)
            break
        return out[:n.value].copy()

    def profile(self, on: bool):
        """Start (clearing earlier records) or stop per-kernel CUDA-event timing."""
        L.check(L.lib().wocr_ctx_profile(self.h, int(bool(on))))

    def profile_report(self):
        """[{kernel, launches, ms, flops, bytes}] of the launches recorded since profile(True)."""
        import json
        buf = ctypes.create_string_buffer(1 << 16)
        L.check(L.lib().wocr_ctx_profile_report(self.h, buf, len(buf)))
        return json.loads(buf.value.decode())

    def profile_launches(self):
        """[{kernel, ms, flops, bytes}] per recorded launch, in launch order."""
        import json
        buf = ctypes.create_string_buffer(1 << 22)
        L.check(L.lib().wocr_ctx_profile_launches(self.h, buf, len(buf)))
        return json.loads(buf.value.decode())

    def close(self):
        if self.h:
            L.lib().wocr_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _Handle:
    kind = 0

    def stats(self) -> Tuple[float, int]:
        """(FLOPs of convolutions/matmuls, kernel launches) of the last run of this handle."""
        f, n = ctypes.c_double(), ctypes.c_int64()
        L.check(L.lib().wocr_last_run_stats(self.h, self.kind, ctypes.byref(f), ctypes.byref(n)))
        return f.value, n.value

    def last_transfer_bytes(self):
        """(bytes host -> device, bytes device -> host) copied by the last call of this handle."""
        a, b = ctypes.c_int64(), ctypes.c_int64()
        L.check(L.lib().wocr_last_transfer_bytes(self.h, self.kind, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value


class Detector(_Handle):
    """`Detector` (src/gpu.rs:1380-1431): the ocrs detection model lowered by Graph::build."""

    kind = 1

    def __init__(self, gpu: Gpu, model: Model):
        self.gpu = gpu
        holder = L.CModelHolder(model)
        h = ctypes.c_void_p()
        L.check(L.lib().wocr_detector_create(gpu.h, holder.ref(), ctypes.byref(h)))
        self.h = h

    def detect_page(self, rgb: np.ndarray, w: int, h: int, threshold: float) -> np.ndarray:
        """RGB bytes of a w x h page -> bit mask [h, ceil(w/32)] u32 (src/gpu.rs:1393-1422)."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        if rgb.size < w * h * 3:
            raise ValueError("rgb smaller than w * h * 3")
        out = np.empty((h, (w + 31) // 32), np.uint32)
        L.check(L.lib().wocr_detect_page(self.h, L.ptr(rgb), w, h, float(threshold), L.ptr(out)))
        return out

    def detect_pages(self, rgb: np.ndarray, threshold: float) -> np.ndarray:
        """n pages [n, h, w, 3] u8 of one size in one pass -> masks [n, h, ceil(w/32)]."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        n, h, w, _ = rgb.shape
        out = np.empty((n, h, (w + 31) // 32), np.uint32)
        L.check(L.lib().wocr_detect_pages(self.h, L.ptr(rgb), n, w, h, float(threshold), L.ptr(out)))
        return out

    def detect_pages_device(self, d_rgb: int, n: int, w: int, h: int, threshold: float, d_mask: int):
        """The same on device pointers, queued on the context stream (no wait)."""
        L.check(L.lib().wocr_detect_pages_device(self.h, ctypes.c_void_p(d_rgb), n, w, h, float(threshold),
                                                 ctypes.c_void_p(d_mask)))

    def detect(self, inp: np.ndarray) -> np.ndarray:
        """The probability map of a [1, 1, h, w] input (src/gpu.rs:1425-1430)."""
        inp = np.ascontiguousarray(inp, np.float32)
        h, w = inp.shape[-2:]
        oh, ow = ctypes.c_int32(), ctypes.c_int32()
        out = np.empty(h * w, np.float32)
        st = L.lib().wocr_detect(self.h, L.ptr(inp), h, w, L.ptr(out), out.size, ctypes.byref(oh), ctypes.byref(ow))
        if st == 8:  # larger output than input: once more with the size it reported
            out = np.empty(oh.value * ow.value, np.float32)
            st = L.lib().wocr_detect(self.h, L.ptr(inp), h, w, L.ptr(out), out.size, ctypes.byref(oh),
                                     ctypes.byref(ow))
        L.check(st)
        return out[: oh.value * ow.value].reshape(oh.value, ow.value)

    def close(self):
        if getattr(self, "h", None):
            L.lib().wocr_detector_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Recognizer(_Handle):
    """`Recognizer` (src/gpu.rs:1433-1603): conv trunk, 2 bidirectional GRU layers, output layer."""

    kind = 2

    def __init__(self, gpu: Gpu, model: Model, lines: int = 8):
        self.gpu = gpu
        holder = L.CModelHolder(model)
        h = ctypes.c_void_p()
        L.check(L.lib().wocr_recognizer_create(gpu.h, holder.ref(), int(lines), ctypes.byref(h)))
        self.h = h

    def dims(self, batches) -> Tuple[int, int, int]:
        bn = (ctypes.c_int32 * len(batches))(*[int(b[1]) for b in batches])
        bw = (ctypes.c_int32 * len(batches))(*[int(b[2]) for b in batches])
        t, n, c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        L.check(L.lib().wocr_recognizer_dims(self.h, bn, bw, len(batches), ctypes.byref(t), ctypes.byref(n),
                                             ctypes.byref(c)))
        return t.value, n.value, c.value

    def recognize(self, batches: Sequence[Tuple[np.ndarray, int, int]], want_logits: bool = True):
        """Batches of (data [n, 1, 64, w] f32, n, w) -> (logits [tmax, ntot, classes] or None,
        tmax, lens, best [tmax, ntot]).  Rows t >= lens[line] of logits/best are unspecified."""
        tmax, ntot, classes = self.dims(batches)
        datas = [np.ascontiguousarray(b[0], np.float32) for b in batches]
        ptrs = (ctypes.c_void_p * len(batches))(*[d.ctypes.data for d in datas])
        bn = (ctypes.c_int32 * len(batches))(*[int(b[1]) for b in batches])
        bw = (ctypes.c_int32 * len(batches))(*[int(b[2]) for b in batches])
        logits = np.empty((tmax, ntot, classes), np.float32) if want_logits else None
        best = np.empty((tmax, ntot), np.uint32)
        lens = (ctypes.c_int32 * ntot)()
        tm = ctypes.c_int32()
        L.check(L.lib().wocr_recognize(self.h, ptrs, bn, bw, len(batches),
                                       L.ptr(logits) if logits is not None else None,
                                       logits.size if logits is not None else 0, lens, L.ptr(best), ctypes.byref(tm)))
        return logits, tm.value, list(lens), best

    def close(self):
        if getattr(self, "h", None):
            L.lib().wocr_recognizer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """A record-then-read list (`wocr_batch`): the reference's command encoder plus
    `Gpu::read_many` (src/gpu.rs:1011-1037).  `NdGraph.argmax_enqueue` / `run_enqueue` queue work
    on the device without waiting; `wait()` waits once and fills every pending result."""

    def __init__(self, gpu: Gpu):
        self.gpu = gpu
        h = ctypes.c_void_p()
        L.check(L.lib().wocr_batch_create(gpu.h, ctypes.byref(h)))
        self.h = h
        self._keep = []      # inputs and outputs that must live until the wait
        self._pending = []

    @property
    def pending(self) -> int:
        return int(L.lib().wocr_batch_pending(self.h))

    def wait(self, timeout_ms: int = 0):
        """Wait (bounded when timeout_ms > 0) and deliver every recorded result."""
        L.check(L.lib().wocr_wait(self.h, int(timeout_ms)))
        for p in self._pending:
            p.done = True
        self._pending = []
        self._keep = []

    def close(self):
        if getattr(self, "h", None):
            L.lib().wocr_batch_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Pending:
    """Results of one enqueued call, valid once its batch has waited (`done`)."""

    def __init__(self, **kw):
        self.done = False
        self.__dict__.update(kw)


class NdGraph(_Handle):
    """`NdGraph` (src/nd.rs:428-1394): the N-D executor with its load-time fusions."""

    kind = 3

    def __init__(self, gpu: Gpu, model: Model, stop_before_softmax: bool = False):
        self.gpu = gpu
        holder = L.CModelHolder(model)
        h = ctypes.c_void_p()
        L.check(L.lib().wocr_ndgraph_create(gpu.h, holder.ref(), int(bool(stop_before_softmax)), ctypes.byref(h)))
        self.h = h
        self._cap = 1 << 20

    def run(self, x: np.ndarray) -> np.ndarray:
        """NdGraph::run (src/nd.rs:834-1195) on a host tensor; the output read back."""
        x = np.ascontiguousarray(x, np.float32)
        shp = (ctypes.c_int64 * x.ndim)(*x.shape)
        oshape = (ctypes.c_int64 * 6)()
        orank = ctypes.c_int32()
        while True:
            out = np.empty(self._cap, np.float32)
            st = L.lib().wocr_ndgraph_run(self.h, L.ptr(x), shp, x.ndim, L.ptr(out), out.size, oshape,
                                          ctypes.byref(orank))
            shape = tuple(oshape[i] for i in range(orank.value))
            if st == 8 and orank.value > 0:
                self._cap = int(np.prod(shape))
                continue
            L.check(st)
            return out[: int(np.prod(shape))].reshape(shape)

    def argmax(self, x: np.ndarray, lse: bool = True):
        """run + arg-max over the last axis per row (ties -> lowest index, src/nd.rs:360-391).
        Returns (best [rows], row_max [rows], row_lse [rows], output shape); with lse=False the
        log-sum-exp is not computed (as the reference's argmax, which gives the classes only)
        and row_lse is None."""
        x = np.ascontiguousarray(x, np.float32)
        shp = (ctypes.c_int64 * x.ndim)(*x.shape)
        cap = max(int(np.prod(x.shape)), 1 << 16)
        while True:
            best = np.empty(cap, np.uint32)
            mx = np.empty(cap, np.float32)
            ls = np.empty(cap, np.float32) if lse else None
            rows = ctypes.c_int64()
            oshape = (ctypes.c_int64 * 6)()
            orank = ctypes.c_int32()
            st = L.lib().wocr_ndgraph_run_argmax(self.h, L.ptr(x), shp, x.ndim, L.ptr(best), L.ptr(mx),
                                                 L.ptr(ls) if lse else None, cap, ctypes.byref(rows), oshape,
                                                 ctypes.byref(orank))
            if st == 8 and rows.value > cap:
                cap = rows.value
                continue
            L.check(st)
            r = rows.value
            shape = tuple(oshape[i] for i in range(orank.value))
            return best[:r], mx[:r], (ls[:r] if lse else None), shape

    def argmax_enqueue(self, batch: "Batch", x: np.ndarray) -> "Pending":
        """NdGraph::run + argmax_record (src/nd.rs:1372-1380): queued on the device, read by
        `batch.wait()`.  Returns a `Pending` whose best / row_max / row_lse ([rows]) and shape
        are filled by the wait."""
        x = np.ascontiguousarray(x, np.float32)
        shp = (ctypes.c_int64 * x.ndim)(*x.shape)
        cap = max(int(np.prod(x.shape)), 1 << 16)
        while True:
            best = np.empty(cap, np.uint32)
            mx = np.empty(cap, np.float32)
            lse = np.empty(cap, np.float32)
            rows = ctypes.c_int64()
            oshape = (ctypes.c_int64 * 6)()
            orank = ctypes.c_int32()
            st = L.lib().wocr_ndgraph_argmax_enqueue(self.h, batch.h, L.ptr(x), shp, x.ndim, L.ptr(best), L.ptr(mx),
                                                     L.ptr(lse), cap, ctypes.byref(rows), oshape, ctypes.byref(orank))
            if st == 8 and rows.value > cap:
                cap = rows.value
                continue
            L.check(st)
            break
        r = rows.value
        pend = Pending(best=best[:r], row_max=mx[:r], row_lse=lse[:r],
                       shape=tuple(oshape[i] for i in range(orank.value)))
        batch._keep += [x, best, mx, lse]
        batch._pending.append(pend)
        return pend

    def ppdet_page(self, rgb: np.ndarray, w: int, h: int, max_side: int, read_map: bool = True):
        """det_input + run on one page (src/bin/ocr-bench.rs:186-200): (prob [oh, ow], to_page).
        With read_map=False the map stays on the device (for db_mask / db_scores) and prob is None."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        ow, oh = ctypes.c_int32(), ctypes.c_int32()
        tp = (ctypes.c_float * 2)()
        prob = None
        if read_map:
            L.check(L.lib().wocr_det_input(self.gpu.h, L.ptr(rgb), w, h, max_side, None, 0, ctypes.byref(ow),
                                           ctypes.byref(oh), tp))
            prob = np.empty((oh.value, ow.value), np.float32)
        L.check(L.lib().wocr_ppdet_page(self.h, L.ptr(rgb), w, h, max_side, L.ptr(prob) if read_map else None,
                                        prob.size if read_map else 0, ctypes.byref(ow), ctypes.byref(oh), tp))
        return prob, (tp[0], tp[1])

    def db_mask(self, thresh: float) -> np.ndarray:
        """The last `ppdet_page` map thresholded on the device (`p > thresh`, src/ppdet.rs:89):
        uint32 [oh, ceil(ow / 32)], bit b of word j = pixel 32 j + b."""
        ow, oh = ctypes.c_int32(), ctypes.c_int32()
        L.check(L.lib().wocr_ppdet_mask(self.h, thresh, None, 0, ctypes.byref(ow), ctypes.byref(oh)))
        bits = np.empty((oh.value, (ow.value + 31) // 32), np.uint32)
        L.check(L.lib().wocr_ppdet_mask(self.h, thresh, L.ptr(bits), bits.size, ctypes.byref(ow), ctypes.byref(oh)))
        return bits

    def db_boxes(self, thresh: float = 0.2, box_thresh: float = 0.45, unclip_ratio: float = 1.4,
                 min_size: float = 3.0) -> np.ndarray:
        """ppdet::boxes (src/ppdet.rs:87-132) of the last `ppdet_page` map, on the device: float32
        [n, 6] boxes [cx, cy, up_x, up_y, width, height] in page coordinates, reading order."""
        n = ctypes.c_int32()
        out = np.zeros((1024, 6), np.float32)
        for _ in range(2):  # again only when the first guess of the capacity was short (status 8)
            st = L.lib().wocr_ppdet_boxes(self.h, thresh, box_thresh, unclip_ratio, min_size, L.ptr(out),
                                          out.shape[0], ctypes.byref(n))
            if st == 8 and n.value > out.shape[0]:
                out = np.zeros((n.value, 6), np.float32)
                continue
            L.check(st)
            break
        return out[:n.value].copy()

    def db_scores(self, rects) -> np.ndarray:
        """`score` (src/ppdet.rs:63-83) of each box [cx, cy, up_x, up_y, width, height] on the last
        `ppdet_page` map, computed on the device: float32 [n]."""
        r = np.ascontiguousarray(np.asarray(rects, np.float32).reshape(-1, 6))
        out = np.empty(len(r), np.float32)
        L.check(L.lib().wocr_ppdet_scores(self.h, L.ptr(r), len(r), L.ptr(out)))
        return out

    @staticmethod
    def det_input(gpu: Gpu, rgb: np.ndarray, w: int, h: int, max_side: int):
        """NdGraph::det_input (src/nd.rs:1353-1369): ([1, 3, oh, ow] f32, to_page factors)."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        ow, oh = ctypes.c_int32(), ctypes.c_int32()
        tp = (ctypes.c_float * 2)()
        L.check(L.lib().wocr_det_input(gpu.h, L.ptr(rgb), w, h, max_side, None, 0, ctypes.byref(ow),
                                       ctypes.byref(oh), tp))
        out = np.empty((1, 3, oh.value, ow.value), np.float32)
        L.check(L.lib().wocr_det_input(gpu.h, L.ptr(rgb), w, h, max_side, L.ptr(out), out.size, ctypes.byref(ow),
                                       ctypes.byref(oh), tp))
        return out, (tp[0], tp[1])

    def close(self):
        if getattr(self, "h", None):
            L.lib().wocr_ndgraph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- host-side greedy CTC (the reference also decodes on the CPU) ----------------------------
def ocrs_decode(best_col: Sequence[int], steps: int, width: int, alphabet: str) -> str:
    """Greedy CTC of src/bin/ocr-bench.rs:62-74 over per-step best classes of one line: blank 0
    dropped, repeats merged, characters starting at t*4 >= width (in the padding) dropped."""
    s, prev = [], 0
    for t in range(steps):
        b = int(best_col[t])
        if b != 0 and b != prev and t * 4 < width:
            s.append(alphabet[b - 1])
        prev = b
    return "".join(s)


class PPPipeline:
    """The PP-OCRv6 page pipeline of the reference's bench (`wocr_pp_*`; src/bin/ocr-bench.rs:
    133-310, 458-585 with PPDET and PPOCR): detection, DB boxes, line images and recognition of
    a page, with the page uploaded once and the map, mask and line batches kept on the device."""

    def __init__(self, gpu: Gpu, det_model: Model, rec_model: Model):
        self.gpu = gpu
        dh, rh = L.CModelHolder(det_model), L.CModelHolder(rec_model)
        h = ctypes.c_void_p()
        L.check(L.lib().wocr_pp_create(gpu.h, dh.ref(), rh.ref(), ctypes.byref(h)))
        self.h = h

    def page(self, rgb, w: int, h: int, max_side: int = 960, db=(0.3, 0.45, 1.4, 3.0), relv: float = 0.1,
             per_batch: int = 16, d_rgb: int = 0):
        """(boxes float32 [n, 6] in reading order, [arg-max classes per step] per line) of an RGB
        page (host array, or d_rgb, a device pointer).  db = (thresh, box_thresh, unclip_ratio,
        min_size); config 4 uses thresh 0.3."""
        src = ctypes.c_void_p(d_rgb) if d_rgb else L.ptr(np.ascontiguousarray(rgb, np.uint8))
        keep = None if d_rgb else rgb
        dbp = np.float32(db)
        n = ctypes.c_int32()
        boxes = np.zeros((256, 6), np.float32)
        cap = 1 << 16
        for _ in range(8):  # again only when a capacity guess was short (status 8)
            best = np.empty(cap, np.uint32)
            steps = np.zeros(boxes.shape[0], np.int32)
            st = L.lib().wocr_pp_page(self.h, src, int(w), int(h), int(max_side), L.ptr(dbp), relv, int(per_batch),
                                      L.ptr(boxes), boxes.shape[0], ctypes.byref(n), L.ptr(best), cap, L.ptr(steps))
            if st == 8 and n.value > boxes.shape[0]:
                boxes = np.zeros((n.value, 6), np.float32)
                continue
            if st == 8:
                cap *= 4
                continue
            break
        L.check(st)
        del keep
        k = n.value
        ends = np.cumsum(steps[:k])
        return boxes[:k].copy(), [best[e - s:e].copy() for e, s in zip(ends, steps[:k])]

    def pages(self, pages, w: int, h: int, max_side: int = 960, db=(0.3, 0.45, 1.4, 3.0), relv: float = 0.1,
              per_batch: int = 16, merge: int = 1, lanes: int = 1, boxes_only: bool = False):
        """Many pages of one size (`wocr_pp_pages`): host arrays [h, w, 3] u8 or device pointers
        (ints).  `lanes` workers on this GPU take pages in turn; each recognises `merge` of its
        pages with one wait.  Returns [(boxes float32 [n, 6], [classes per step] per line)] per
        page, equal to `page()` page by page.  `self.last_bytes` = (H2D, D2H) bytes."""
        n = len(pages)
        ptrs = (ctypes.c_void_p * max(n, 1))()
        keep = []
        for k, pg in enumerate(pages):
            if isinstance(pg, (int, np.integer)):
                ptrs[k] = int(pg)
            else:
                a = np.ascontiguousarray(pg, np.uint8)
                keep.append(a)
                ptrs[k] = a.ctypes.data
        ws = np.full(max(n, 1), w, np.int32)
        hs = np.full(max(n, 1), h, np.int32)
        dbp = np.float32(db)
        nl = np.zeros(max(n, 1), np.int32)
        byts = np.zeros(2, np.int64)
        box_cap = getattr(self, "_box_cap", 1024 * max(n, 1))
        cap = getattr(self, "_cap", 1 << 18)
        for _ in range(8):  # again only when a capacity guess was short (status 8)
            boxes = np.zeros((box_cap, 6), np.float32)
            best = np.empty(0 if boxes_only else cap, np.uint32)
            steps = np.zeros(box_cap, np.int32)
            st = L.lib().wocr_pp_pages(self.h, ptrs, L.ptr(ws), L.ptr(hs), n, int(max_side), L.ptr(dbp), relv,
                                       int(per_batch), int(merge), int(lanes), L.ptr(boxes), box_cap, L.ptr(nl),
                                       None if boxes_only else L.ptr(best), 0 if boxes_only else cap,
                                       None if boxes_only else L.ptr(steps), L.ptr(byts))
            if st == 8 and int(nl[:n].sum()) > box_cap:
                box_cap = int(nl[:n].sum()) * 2
                continue
            if st == 8:
                cap *= 4
                continue
            break
        L.check(st)
        self._box_cap, self._cap = box_cap, cap
        self.last_bytes = (int(byts[0]), int(byts[1]))
        del keep
        out, b0, l0, o = [], 0, 0, 0
        for k in range(n):
            m = int(nl[k])
            bx = boxes[b0:b0 + m].copy()
            lines = []
            if not boxes_only:
                for i in range(m):
                    t = int(steps[l0 + i])
                    lines.append(best[o:o + t].copy())
                    o += t
            out.append((bx, lines))
            b0 += m
            l0 += m
        return out

    def launches(self) -> int:
        """Kernels launched so far by every lane of this pipeline."""
        return int(L.lib().wocr_pp_launches(self.h))

    def texts(self, rgb, w: int, h: int, chars: List[str], **kw) -> List[str]:
        """The page's text lines in reading order (`Dictionary::decode` of each line)."""
        _, bests = self.page(rgb, w, h, **kw)
        return [pp_decode(b, chars) for b in bests]

    def close(self):
        if self.h:
            L.lib().wocr_pp_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def text_lines(words) -> List[List[int]]:
    """ocrs' find_text_lines as the library restates it (`wocr_text_lines`, host code): the word
    indices of each line (left to right), lines in reading order."""
    r = np.ascontiguousarray(np.asarray(words, np.float32).reshape(-1, 6))
    n = len(r)
    order = np.zeros(max(n, 1), np.int32)
    lens = np.zeros(max(n, 1), np.int32)
    nl = ctypes.c_int32()
    L.check(L.lib().wocr_text_lines(L.ptr(r), n, L.ptr(order), L.ptr(lens), ctypes.byref(nl)))
    out, o = [], 0
    for k in range(nl.value):
        out.append(order[o:o + lens[k]].tolist())
        o += int(lens[k])
    return out


def pad_line(words, relv: float = 0.15, relend: float = 0.1) -> np.ndarray:
    """One line's words padded as src/bin/ocr-bench.rs:534-558 pads them (`wocr_pad_line`)."""
    r = np.array(np.asarray(words, np.float32).reshape(-1, 6), np.float32, copy=True)
    L.check(L.lib().wocr_pad_line(L.ptr(r), len(r), relv, relend))
    return r


class OcrsPipeline:
    """The ocrs page pipeline of the reference's bench (`wocr_ocrs_*`; src/bin/ocr-bench.rs:
    458-585 without DET / REC): detection, word rectangles, text lines, padding, line images and
    recognition, with the pages, masks and line images kept on the device."""

    def __init__(self, gpu: Gpu, det_model: Model, rec_model: Model):
        self.gpu = gpu
        dh, rh = L.CModelHolder(det_model), L.CModelHolder(rec_model)
        h = ctypes.c_void_p()
        L.check(L.lib().wocr_ocrs_create(gpu.h, dh.ref(), rh.ref(), ctypes.byref(h)))
        self.h = h

    def pages(self, pages, w: int, h: int, threshold: float = 0.5, relv: float = 0.15, relend: float = 0.1,
              merge: int = 1, lanes: int = 1):
        """Pages of one size (host arrays [h, w, 3] u8 or device pointers).  Returns per page a
        list of lines in reading order, each (padded words float32 [k, 6], image width W, arg-max
        classes of its steps).  `self.last_bytes` = (H2D, D2H) bytes."""
        n = len(pages)
        ptrs = (ctypes.c_void_p * max(n, 1))()
        keep = []
        for k, pg in enumerate(pages):
            if isinstance(pg, (int, np.integer)):
                ptrs[k] = int(pg)
            else:
                a = np.ascontiguousarray(pg, np.uint8)
                keep.append(a)
                ptrs[k] = a.ctypes.data
        nl = np.zeros(max(n, 1), np.int32)
        byts = np.zeros(2, np.int64)
        lcap = getattr(self, "_lcap", 256 * max(n, 1))
        wcap = getattr(self, "_wcap", 2048 * max(n, 1))
        cap = getattr(self, "_cap", 1 << 18)
        for _ in range(8):  # again only when a capacity guess was short (status 8)
            lw = np.zeros(lcap, np.int32)
            widths = np.zeros(lcap, np.int32)
            steps = np.zeros(lcap, np.int32)
            words = np.zeros((wcap, 6), np.float32)
            best = np.empty(cap, np.uint32)
            st = L.lib().wocr_ocrs_pages(self.h, ptrs, n, int(w), int(h), float(threshold), relv, relend, int(merge),
                                         int(lanes), L.ptr(nl), L.ptr(lw), lcap, L.ptr(words), wcap, L.ptr(widths),
                                         L.ptr(steps), L.ptr(best), cap, L.ptr(byts))
            if st == 8:
                lcap, wcap, cap = lcap * 4, wcap * 4, cap * 4
                continue
            break
        L.check(st)
        self._lcap, self._wcap, self._cap = lcap, wcap, cap
        self.last_bytes = (int(byts[0]), int(byts[1]))
        del keep
        out, li, wi, o = [], 0, 0, 0
        for k in range(n):
            lines = []
            for _ in range(int(nl[k])):
                kw, t = int(lw[li]), int(steps[li])
                lines.append((words[wi:wi + kw].copy(), int(widths[li]), best[o:o + t].copy()))
                wi += kw
                o += t
                li += 1
            out.append(lines)
        return out

    def launches(self) -> int:
        """Kernels launched so far by every lane of this pipeline."""
        return int(L.lib().wocr_ocrs_launches(self.h))

    def texts(self, pages, w: int, h: int, alphabet: str, **kw) -> List[List[str]]:
        """Each page's text lines (greedy CTC of src/bin/ocr-bench.rs:62-74)."""
        return [[ocrs_decode(b, len(b), W, alphabet) for _, W, b in lines] for lines in self.pages(pages, w, h, **kw)]

    def close(self):
        if self.h:
            L.lib().wocr_ocrs_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def load_pp_dictionary(path: str) -> List[str]:
    """`Dictionary::load` (src/ppocr.rs:10-16): class 0 the blank, then the file's lines in order
    (split as Rust's `str::lines` splits: at "\n", a "\r" before it dropped, no empty line after
    a final newline), then the space."""
    with open(path, encoding="utf-8") as f:
        text = f.read()
    lines = text.split("\n")
    if lines and lines[-1] == "":
        lines.pop()
    return [""] + [ln[:-1] if ln.endswith("\r") else ln for ln in lines] + [" "]


def pp_decode(best: Sequence[int], chars: List[str]) -> str:
    """`Dictionary::decode` (src/ppocr.rs:23-33): repeats merged, blanks dropped."""
    out, prev = [], 0
    for c in best:
        c = int(c)
        if c != 0 and c != prev:
            out.append(chars[c] if c < len(chars) else "")
        prev = c
    return "".join(out)
