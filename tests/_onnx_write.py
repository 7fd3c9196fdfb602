"""A minimal writer of ONNX ModelProto bytes (the protobuf wire format, onnx.proto field numbers)
for the loader tests: the `onnx` package is not installed, and the reference's models are not
present, so the tests write their own files from the synthetic `Model`s.  Options vary the
encodings a reader must accept: raw_data or typed value fields, packed or one-per-field
repeated numbers, attributes with or without their type, and fields the reader must skip."""
import struct

import numpy as np


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1  # int64 as two's complement, as protobuf encodes negative varints
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint(field << 3 | wire)


def _len(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _str(field: int, s: str) -> bytes:
    return _len(field, s.encode())


def _ints(field: int, vals, packed: bool) -> bytes:
    if packed:
        return _len(field, b"".join(_varint(int(v)) for v in vals)) if len(vals) else b""
    return b"".join(_key(field, 0) + _varint(int(v)) for v in vals)


def _floats(field: int, vals, packed: bool) -> bytes:
    if packed:
        return _len(field, b"".join(struct.pack("<f", float(v)) for v in vals)) if len(vals) else b""
    return b"".join(_key(field, 5) + struct.pack("<f", float(v)) for v in vals)


def tensor(name, arr: np.ndarray, dtype: int, raw=True, packed=True, named=True, extra=False) -> bytes:
    """TensorProto: dims (1), data_type (2), float_data (4), int64_data (7), name (8),
    raw_data (9); with `extra`, a doc_string (12) and an int32_data field (5) to skip."""
    arr = np.asarray(arr, np.float32 if dtype == 1 else np.int64)
    out = _ints(1, list(arr.shape), packed) + _key(2, 0) + _varint(dtype)
    if raw:
        out += _len(9, arr.astype("<f4" if dtype == 1 else "<i8").tobytes())
    elif dtype == 1:
        out += _floats(4, arr.ravel().tolist(), packed)
    else:
        out += _ints(7, arr.ravel().tolist(), packed)
    if named:
        out += _str(8, name)
    if extra:
        out += _str(12, "skipped") + _ints(5, [1, 2, 3], True)
    return out


def attr(name, v, typed=True, packed=True) -> bytes:
    """AttributeProto: name (1), f (2), i (3), s (4), floats (7), ints (8), type (20)."""
    out = _str(1, name)
    if isinstance(v, bool) or isinstance(v, (int, np.integer)):
        out += _key(3, 0) + _varint(int(v))
        t = 2
    elif isinstance(v, (float, np.floating)):
        out += _key(2, 5) + struct.pack("<f", float(v))
        t = 1
    elif isinstance(v, str):
        out += _str(4, v)
        t = 3
    elif all(isinstance(x, (int, np.integer)) for x in v):
        out += _ints(8, list(v), packed)
        t = 7
    else:
        out += _floats(7, list(v), packed)
        t = 6
    if typed:
        out += _key(20, 0) + _varint(t)
    return out


def node(op, inputs, outputs, attrs, typed=True, packed=True) -> bytes:
    """NodeProto: input (1), output (2), name (3), op_type (4), attribute (5), domain (7)."""
    out = b"".join(_str(1, s) for s in inputs) + b"".join(_str(2, s) for s in outputs)
    out += _str(3, f"{op}_node") + _str(4, op) + _str(7, "")
    out += b"".join(_len(5, attr(k, v, typed, packed)) for k, v in attrs.items())
    return out


def value_info(name) -> bytes:
    """ValueInfoProto: name (1) and a type (2) to skip."""
    return _str(1, name) + _len(2, _len(1, _key(1, 0) + _varint(1)))


def model(m, raw=True, packed=True, typed=True, inits_as_inputs=False, constants=(), extra=False) -> bytes:
    """ModelProto bytes of `m`.  `constants`: initializer names written as Constant nodes (before
    the other nodes) instead of initializers.  `extra`: fields the reader must skip (producer,
    opset, doc strings, value_info)."""
    g = b""
    for name in constants:
        dt, arr = (1, m.weights[name]) if name in m.weights else (7, m.ints[name])
        t = tensor("", arr, dt, raw, packed, named=False)
        g += _len(1, node("Constant", [], [name], {}, typed, packed) + _len(5, _str(1, "value") + _len(5, t) +
                                                                      _key(20, 0) + _varint(4)))
    for n in m.nodes:
        g += _len(1, node(n.op, n.inputs, n.outputs, n.attrs, typed, packed))
    g += _str(2, "graph")
    for name, w in m.weights.items():
        if name not in constants:
            g += _len(5, tensor(name, w, 1, raw, packed, extra=extra))
    for name, v in m.ints.items():
        if name not in constants:
            g += _len(5, tensor(name, v, 7, raw, packed, extra=extra))
    ins = ([k for k in m.weights if k not in constants] if inits_as_inputs else []) + [m.input]
    g += b"".join(_len(11, value_info(s)) for s in ins)
    g += _len(12, value_info(m.output))
    if extra:
        g += _str(10, "graph doc") + _len(13, value_info("intermediate"))
    out = _key(1, 0) + _varint(8)
    if extra:
        out += _str(2, "writer") + _str(3, "1") + _len(8, _str(1, "") + _key(2, 0) + _varint(17))
    return out + _len(7, g)
