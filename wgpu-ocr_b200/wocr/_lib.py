"""ctypes binding of libwocr.so (include/wocr.h).

The library is loaded from this directory only (it is built in-tree by
`wgpu-ocr_b200/build.py`); there is no other implementation to fall back to, so a missing or
unloadable library raises immediately.
"""
from __future__ import annotations

import ctypes
import os
from typing import List

import numpy as np

from .model import Model

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwocr.so")

c_i32, c_i64, c_f32, c_f64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_double
c_void_p, c_char_p, c_size_t = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t
P = ctypes.POINTER


class Attr(ctypes.Structure):
    _fields_ = [("name", c_char_p), ("kind", c_i32), ("i", c_i64), ("f", c_f32), ("s", c_char_p),
                ("ints", P(c_i64)), ("floats", P(c_f32)), ("count", c_i64)]


class CNode(ctypes.Structure):
    _fields_ = [("op", c_char_p), ("inputs", P(c_char_p)), ("n_inputs", c_i32), ("outputs", P(c_char_p)),
                ("n_outputs", c_i32), ("attrs", P(Attr)), ("n_attrs", c_i32)]


class Init(ctypes.Structure):
    _fields_ = [("name", c_char_p), ("dtype", c_i32), ("dims", P(c_i64)), ("rank", c_i32), ("data", c_void_p)]


class CModel(ctypes.Structure):
    _fields_ = [("nodes", P(CNode)), ("n_nodes", c_i32), ("inits", P(Init)), ("n_inits", c_i32),
                ("input", c_char_p), ("output", c_char_p)]


ATTR_INT, ATTR_FLOAT, ATTR_STRING, ATTR_INTS, ATTR_FLOATS = 1, 2, 3, 4, 5

# status codes of include/wocr.h
STATUS = {0: "OK", 1: "INVALID", 2: "UNSUPPORTED", 3: "SHAPE", 4: "OOM", 5: "CUDA", 6: "TIMEOUT", 7: "MISSING",
          8: "CAPACITY"}


class WocrError(RuntimeError):
    """A failing libwocr call: `code` is the status, the message is wocr_last_error()."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS.get(code, code)}: {message}")
        self.code = code
        self.message = message


_lib = None

# (name, restype, argtypes)
_SIGS = [
    ("wocr_last_error", c_char_p, []),
    ("wocr_ctx_create", c_i32, [c_i32, c_i32, P(c_void_p)]),
    ("wocr_ctx_destroy", None, [c_void_p]),
    ("wocr_ctx_describe", c_i32, [c_void_p, c_char_p, c_i32]),
    ("wocr_ctx_stream", c_void_p, [c_void_p]),
    ("wocr_ctx_sync", c_i32, [c_void_p, c_i32]),
    ("wocr_ctx_pool_bytes", c_i64, [c_void_p]),
    ("wocr_ctx_launches", c_i64, [c_void_p]),
    ("wocr_ctx_profile", c_i32, [c_void_p, c_i32]),
    ("wocr_ctx_profile_report", c_i32, [c_void_p, c_char_p, c_i32]),
    ("wocr_ctx_profile_launches", c_i32, [c_void_p, c_char_p, c_i32]),
    ("wocr_host_alloc", c_i32, [c_size_t, P(c_void_p)]),
    ("wocr_host_free", None, [c_void_p]),
    ("wocr_detector_create", c_i32, [c_void_p, P(CModel), P(c_void_p)]),
    ("wocr_detector_destroy", None, [c_void_p]),
    ("wocr_detect_page", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_f32, c_void_p]),
    ("wocr_detect", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_void_p, c_i64, P(c_i32), P(c_i32)]),
    ("wocr_detect_pages", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_f32, c_void_p]),
    ("wocr_detect_pages_device", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_f32, c_void_p]),
    ("wocr_recognizer_create", c_i32, [c_void_p, P(CModel), c_i32, P(c_void_p)]),
    ("wocr_recognizer_destroy", None, [c_void_p]),
    ("wocr_recognizer_dims", c_i32, [c_void_p, P(c_i32), P(c_i32), c_i32, P(c_i32), P(c_i32), P(c_i32)]),
    ("wocr_recognize", c_i32, [c_void_p, P(c_void_p), P(c_i32), P(c_i32), c_i32, c_void_p, c_i64, P(c_i32),
                               c_void_p, P(c_i32)]),
    ("wocr_ndgraph_create", c_i32, [c_void_p, P(CModel), c_i32, P(c_void_p)]),
    ("wocr_ndgraph_destroy", None, [c_void_p]),
    ("wocr_ndgraph_run", c_i32, [c_void_p, c_void_p, P(c_i64), c_i32, c_void_p, c_i64, P(c_i64), P(c_i32)]),
    ("wocr_ndgraph_run_argmax", c_i32, [c_void_p, c_void_p, P(c_i64), c_i32, c_void_p, c_void_p, c_void_p, c_i64,
                                        P(c_i64), P(c_i64), P(c_i32)]),
    ("wocr_argmax_rows_noalloc", c_i32, [c_void_p, c_void_p, c_i64, c_i64, c_void_p, c_void_p, c_void_p]),
    ("wocr_det_input", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_void_p, c_i64, P(c_i32), P(c_i32),
                               P(c_f32)]),
    ("wocr_ppdet_page", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_void_p, c_i64, P(c_i32), P(c_i32),
                                P(c_f32)]),
    ("wocr_last_run_stats", c_i32, [c_void_p, c_i32, P(c_f64), P(c_i64)]),
    ("wocr_last_transfer_bytes", c_i32, [c_void_p, c_i32, P(c_i64), P(c_i64)]),
    ("wocr_word_rects", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_i32, c_f32, c_f32, c_f32, c_void_p, c_i64,
                                c_void_p]),
    ("wocr_pp_create", c_i32, [c_void_p, P(CModel), P(CModel), P(c_void_p)]),
    ("wocr_pp_destroy", None, [c_void_p]),
    ("wocr_pp_launches", c_i64, [c_void_p]),
    ("wocr_pp_page", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_void_p, c_f32, c_i32, c_void_p, c_i32,
                             P(c_i32), c_void_p, c_i64, c_void_p]),
    ("wocr_ppdet_boxes", c_i32, [c_void_p, c_f32, c_f32, c_f32, c_f32, c_void_p, c_i32, P(c_i32)]),
    ("wocr_db_boxes", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_void_p, c_f32, c_f32, c_f32, c_f32, c_void_p,
                              c_i32, P(c_i32)]),
    ("wocr_ppdet_mask", c_i32, [c_void_p, c_f32, c_void_p, c_i64, P(c_i32), P(c_i32)]),
    ("wocr_ppdet_scores", c_i32, [c_void_p, c_void_p, c_i32, c_void_p]),
    ("wocr_model_load", c_i32, [c_char_p, P(P(CModel))]),
    ("wocr_model_parse", c_i32, [c_void_p, c_i64, P(P(CModel))]),
    ("wocr_model_free", None, [P(CModel)]),
    ("wocr_batch_create", c_i32, [c_void_p, P(c_void_p)]),
    ("wocr_batch_destroy", None, [c_void_p]),
    ("wocr_batch_pending", c_i64, [c_void_p]),
    ("wocr_ndgraph_run_enqueue", c_i32, [c_void_p, c_void_p, c_void_p, P(c_i64), c_i32, c_void_p, c_i64, P(c_i64),
                                         P(c_i32)]),
    ("wocr_ndgraph_argmax_enqueue", c_i32, [c_void_p, c_void_p, c_void_p, P(c_i64), c_i32, c_void_p, c_void_p,
                                            c_void_p, c_i64, P(c_i64), P(c_i64), P(c_i32)]),
    ("wocr_wait", c_i32, [c_void_p, c_i32]),
    ("wocr_pp_pages", c_i32, [c_void_p, c_void_p, c_void_p, c_void_p, c_i32, c_i32, c_void_p, c_f32, c_i32, c_i32,
                              c_i32, c_void_p, c_i64, c_void_p, c_void_p, c_i64, c_void_p, c_void_p]),
    ("wocr_text_lines", c_i32, [c_void_p, c_i32, c_void_p, c_void_p, P(c_i32)]),
    ("wocr_pad_line", c_i32, [c_void_p, c_i32, c_f32, c_f32]),
    ("wocr_ocrs_lines", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_void_p, c_void_p, c_i32, c_void_p, c_i64,
                                c_void_p, c_void_p, c_void_p, c_void_p, P(c_i32), P(c_i64)]),
    ("wocr_ocrs_create", c_i32, [c_void_p, P(CModel), P(CModel), P(c_void_p)]),
    ("wocr_ocrs_destroy", None, [c_void_p]),
    ("wocr_ocrs_launches", c_i64, [c_void_p]),
    ("wocr_ocrs_pages", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_i32, c_f32, c_f32, c_f32, c_i32, c_i32, c_void_p,
                                c_void_p, c_i64, c_void_p, c_i64, c_void_p, c_void_p, c_void_p, c_i64, c_void_p]),
    ("wocr_pp_lines", c_i32, [c_void_p, c_void_p, c_i32, c_i32, c_void_p, c_i32, c_i32, c_void_p, c_i64, c_void_p,
                              c_void_p, c_void_p, P(c_i32), P(c_i64)]),
]

EXPORTS = [s[0] for s in _SIGS]


def lib():
    """Load libwocr.so (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python wgpu-ocr_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int):
    if status != 0:
        msg = lib().wocr_last_error()
        raise WocrError(int(status), msg.decode() if msg else "")


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class CModelHolder:
    """A `Model` flattened into the wocr_model structs; keeps every buffer alive."""

    def __init__(self, m: Model):
        keep: List = []

        def cs(s: str):
            b = s.encode()
            keep.append(b)
            return b

        def strs(names):
            arr = (c_char_p * max(len(names), 1))(*[cs(n) for n in names])
            keep.append(arr)
            return arr

        nodes = (CNode * max(len(m.nodes), 1))()
        for k, n in enumerate(m.nodes):
            attrs = (Attr * max(len(n.attrs), 1))()
            for q, (name, v) in enumerate(n.attrs.items()):
                a = attrs[q]
                a.name = cs(name)
                if isinstance(v, bool) or isinstance(v, (int, np.integer)):
                    a.kind, a.i = ATTR_INT, int(v)
                elif isinstance(v, (float, np.floating)):
                    a.kind, a.f = ATTR_FLOAT, float(v)
                elif isinstance(v, str):
                    a.kind, a.s = ATTR_STRING, cs(v)
                elif all(isinstance(x, (int, np.integer)) for x in v):
                    arr = np.asarray(v, np.int64)
                    keep.append(arr)
                    a.kind, a.ints, a.count = ATTR_INTS, arr.ctypes.data_as(P(c_i64)), len(arr)
                else:
                    arr = np.asarray(v, np.float32)
                    keep.append(arr)
                    a.kind, a.floats, a.count = ATTR_FLOATS, arr.ctypes.data_as(P(c_f32)), len(arr)
            keep.append(attrs)
            nodes[k].op = cs(n.op)
            nodes[k].inputs = strs(n.inputs)
            nodes[k].n_inputs = len(n.inputs)
            nodes[k].outputs = strs(n.outputs)
            nodes[k].n_outputs = len(n.outputs)
            nodes[k].attrs = attrs
            nodes[k].n_attrs = len(n.attrs)
        items = [(k, v, 1) for k, v in m.weights.items()] + [(k, v, 7) for k, v in m.ints.items()]
        inits = (Init * max(len(items), 1))()
        for q, (name, v, dt) in enumerate(items):
            arr = np.ascontiguousarray(v, np.float32 if dt == 1 else np.int64)
            dims = np.asarray(arr.shape, np.int64)
            keep += [arr, dims]
            inits[q].name = cs(name)
            inits[q].dtype = dt
            inits[q].dims = dims.ctypes.data_as(P(c_i64))
            inits[q].rank = arr.ndim
            inits[q].data = arr.ctypes.data
        keep += [nodes, inits]
        self.c = CModel(nodes, len(m.nodes), inits, len(items), cs(m.input), cs(m.output))
        self._keep = keep

    def ref(self):
        return ctypes.byref(self.c)
