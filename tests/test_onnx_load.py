"""The C++ ONNX reader (`wocr_model_load` / `wocr_model_parse`) against the reference loader's
semantics (src/onnx.rs:57-123): the synthetic models of every benchmark configuration written
as ONNX bytes in several encodings read back to the same Model; Constant nodes fold into the
initializers; the graph input and output rules; the loader's errors.  CPU only: loading needs
no GPU."""
import numpy as np
import pytest

import wocr
from wocr import synth
from wocr.model import Model, Node

from _onnx_write import _key, _len, _str, _varint, model, node, tensor, value_info


def same(a: Model, b: Model):
    assert (a.input, a.output) == (b.input, b.output)
    assert len(a.nodes) == len(b.nodes)
    for x, y in zip(a.nodes, b.nodes):
        assert (x.op, x.inputs, x.outputs) == (y.op, y.inputs, y.outputs)
        assert x.attrs.keys() == y.attrs.keys(), (x.op, x.attrs, y.attrs)
        for k in x.attrs:
            u, v = x.attrs[k], y.attrs[k]
            if isinstance(u, float) or (isinstance(u, list) and u and isinstance(u[0], float)):
                np.testing.assert_array_equal(np.float32(u), np.float32(v))
            else:
                assert u == v, (x.op, k, u, v)
    assert a.weights.keys() == b.weights.keys()
    for k in a.weights:
        assert a.weights[k].shape == b.weights[k].shape, k
        np.testing.assert_array_equal(a.weights[k], b.weights[k])
    assert a.ints.keys() == b.ints.keys()
    for k in a.ints:
        np.testing.assert_array_equal(np.asarray(a.ints[k], np.int64).ravel(), np.asarray(b.ints[k]).ravel())


MODELS = {"ocrs_det": synth.ocrs_det_model, "ocrs_rec": synth.ocrs_rec_model, "pp_rec": synth.pp_rec_model,
          "pp_det": synth.pp_det_model}


@pytest.fixture(scope="module", params=list(MODELS))
def synth_model(request):
    return MODELS[request.param]()


@pytest.mark.parametrize("raw,packed,typed,extra", [(True, True, True, False), (False, False, False, True),
                                                    (False, True, True, True)])
def test_round_trip(synth_model, raw, packed, typed, extra):
    """raw_data or float_data / int64_data, packed or not, typed attributes or not, fields to
    skip; the initializers also listed as graph inputs (older exporters do), so the input is the
    first one that is not a weight."""
    data = model(synth_model, raw=raw, packed=packed, typed=typed, inits_as_inputs=True, extra=extra)
    same(wocr.parse_onnx(data), synth_model)


def test_load_file(tmp_path, synth_model):
    p = tmp_path / "m.onnx"
    p.write_bytes(model(synth_model))
    same(wocr.load_onnx(str(p)), synth_model)
    with pytest.raises(wocr.WocrError, match="cannot open"):
        wocr.load_onnx(str(tmp_path / "missing.onnx"))


def test_constants_fold_into_initializers():
    """Constant nodes (a float tensor and an int64 list) become initializers named after their
    output, and the nodes are dropped (src/onnx.rs:105-112)."""
    m = synth.pp_rec_model()
    ints = list(m.ints)[:2]
    fl = list(m.weights)[:1]
    assert ints, "the PP model has integer constants"
    got = wocr.parse_onnx(model(m, constants=ints + fl))
    assert not any(n.op == "Constant" for n in got.nodes)
    assert set(got.ints) == set(m.ints) and set(got.weights) == set(m.weights)
    same(got, m)


def _graph(*parts) -> bytes:
    return _key(1, 0) + _varint(8) + _len(7, b"".join(parts))


def test_input_output_rules_and_int64_lists():
    """The graph input is the first input that is not a float weight (an int64 list does not
    count), the output the first graph output; an int64 list keeps its length whatever its dims
    say, and non-float, non-int64 initializers are dropped."""
    w = tensor("w", np.ones((2, 2), np.float32), 1)
    shape = tensor("shape", np.array([1, 2, 3], np.int64), 7)
    odd = _str(8, "odd") + _key(1, 0) + _varint(5) + _key(2, 0) + _varint(7) + _key(7, 0) + _varint(4)
    half = _str(8, "half") + _key(1, 0) + _varint(2) + _key(2, 0) + _varint(10)  # float16: dropped
    n = _len(1, node("Reshape", ["x", "shape"], ["y"], {}))
    data = _graph(n, _len(5, w), _len(5, shape), _len(5, odd), _len(5, half), _len(11, value_info("w")),
                  _len(11, value_info("shape")), _len(11, value_info("x")), _len(12, value_info("y")),
                  _len(12, value_info("z")))
    got = wocr.parse_onnx(data)
    assert got.input == "shape" and got.output == "y"
    assert list(got.ints["odd"].ravel()) == [4] and "half" not in got.weights and "half" not in got.ints
    assert list(got.ints["shape"].ravel()) == [1, 2, 3]
    assert got.weights["w"].shape == (2, 2)


def test_attribute_kinds():
    """Typed and untyped attributes, negative ints, an empty list, a tensor attribute on an op
    other than Constant (read as an empty int list, as Node::ints sees it)."""
    attrs = {"axis": -1, "alpha": 0.25, "mode": "nearest", "pads": [1, -2, 3, 4], "scales": [1.0, 2.5],
             "empty": []}
    for typed in (True, False):
        n = node("Op", ["x"], ["y"], attrs, typed=typed)
        n += _len(5, _str(1, "value") + _len(5, tensor("", np.zeros(2, np.float32), 1)) + _key(20, 0) + _varint(4))
        got = wocr.parse_onnx(_graph(_len(1, n), _len(11, value_info("x")), _len(12, value_info("y"))))
        a = got.nodes[0].attrs
        assert a["axis"] == -1 and a["mode"] == "nearest" and a["pads"] == [1, -2, 3, 4]
        assert np.float32(a["alpha"]) == np.float32(0.25) and np.float32(a["scales"]).tolist() == [1.0, 2.5]
        assert a["empty"] == [] and a["value"] == []


@pytest.mark.parametrize("data,msg", [
    (b"", "model has no graph"),
    (_key(1, 0) + _varint(8), "model has no graph"),
    (_graph(_len(11, value_info("w")), _len(5, tensor("w", np.ones(2, np.float32), 1)), _len(12, value_info("y"))),
     "no graph input"),
    (_graph(_len(11, value_info("x"))), "no graph output"),
    (_graph(_len(5, _str(8, "w") + _key(1, 0) + _varint(4) + _key(2, 0) + _varint(1) + _len(4, b"\0" * 12)),
            _len(11, value_info("x")), _len(12, value_info("y"))), 'Some\\("w"\\): 3 values for 4'),
    (_graph(_len(5, _str(8, "w") + _key(1, 0) + _varint(-2) + _key(2, 0) + _varint(1)), _len(11, value_info("x")),
            _len(12, value_info("y"))), "negative dimension"),
    (_key(7, 2) + _varint(50) + b"\x0a", "truncated"),
])
def test_errors(data, msg):
    with pytest.raises(wocr.WocrError, match=msg):
        wocr.parse_onnx(data)


def test_loaded_model_builds_the_cpu_checker_graph():
    """A loaded model runs through the CPU oracle's ONNX interpreter like the original."""
    from oracle import ref

    m = synth.ocrs_det_model()
    got = wocr.parse_onnx(model(m, raw=False, packed=False))
    x = np.random.default_rng(0).standard_normal((1, 1, 64, 48)).astype(np.float32)
    np.testing.assert_array_equal(ref.run_onnx(got, x), ref.run_onnx(m, x))
