"""ONNX files read by the library's C++ loader (`wocr_model_load`, `wocr_model_parse`; the
semantics of the reference's `Onnx::load`, src/onnx.rs:57-123) and turned into a `Model`."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from .model import Model, Node


def _to_model(cm: L.CModel) -> Model:
    def names(p, n):
        return [p[k].decode() for k in range(n)]

    nodes = []
    for k in range(cm.n_nodes):
        n = cm.nodes[k]
        attrs = {}
        for q in range(n.n_attrs):
            a = n.attrs[q]
            name = a.name.decode()
            if a.kind == L.ATTR_INT:
                attrs[name] = int(a.i)
            elif a.kind == L.ATTR_FLOAT:
                attrs[name] = float(a.f)
            elif a.kind == L.ATTR_STRING:
                attrs[name] = a.s.decode()
            elif a.kind == L.ATTR_INTS:
                attrs[name] = [int(a.ints[j]) for j in range(a.count)]
            elif a.kind == L.ATTR_FLOATS:
                attrs[name] = [float(a.floats[j]) for j in range(a.count)]
        nodes.append(Node(n.op.decode(), names(n.inputs, n.n_inputs), names(n.outputs, n.n_outputs), attrs))
    weights, ints = {}, {}
    for k in range(cm.n_inits):
        t = cm.inits[k]
        dims = tuple(int(t.dims[j]) for j in range(t.rank))
        count = int(np.prod(dims)) if dims else 1
        ctype = ctypes.c_float if t.dtype == 1 else ctypes.c_int64
        vals = np.ctypeslib.as_array((ctype * count).from_address(t.data)).copy() if count else np.zeros(0)
        if t.dtype == 1:
            weights[t.name.decode()] = vals.astype(np.float32).reshape(dims)
        else:
            ints[t.name.decode()] = vals.astype(np.int64).reshape(dims)
    return Model(nodes, weights, ints, cm.input.decode(), cm.output.decode())


def _take(status: int, out) -> Model:
    L.check(status)
    try:
        return _to_model(out.contents)
    finally:
        L.lib().wocr_model_free(out)


def load_onnx(path: str) -> Model:
    """An .onnx file as the reference's Onnx::load reads it (src/onnx.rs:88-123)."""
    out = ctypes.POINTER(L.CModel)()
    return _take(L.lib().wocr_model_load(str(path).encode(), ctypes.byref(out)), out)


def parse_onnx(data: bytes) -> Model:
    """The same from the bytes of an ONNX ModelProto."""
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    out = ctypes.POINTER(L.CModel)()
    return _take(L.lib().wocr_model_parse(buf, len(data), ctypes.byref(out)), out)
