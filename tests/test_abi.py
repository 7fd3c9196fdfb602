"""The C-ABI library: it loads, exports every entry point include/wocr.h declares, and reports
errors as status codes with a message (no GPU needed)."""
import ctypes
import os
import re

import pytest

import wocr
from wocr import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "wocr.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wocr_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = wocr.lib()
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), f"{n} declared in wocr.h but not exported"
    # and the Python binding declares a signature for each of them
    assert set(names) == set(_lib.EXPORTS)


def test_library_is_the_in_tree_build():
    assert os.path.dirname(wocr.LIB_PATH) == os.path.join(ROOT, "wgpu-ocr_b200", "wocr")


def test_null_arguments_are_status_codes():
    L = wocr.lib()
    assert L.wocr_ctx_create(0, 8, None) == 1              # WOCR_ERR_INVALID
    assert b"null" in L.wocr_last_error()
    assert L.wocr_ctx_sync(None, 0) == 1
    assert L.wocr_last_run_stats(None, 1, None, None) == 1
    L.wocr_ctx_destroy(None)                                 # no-op, no crash
    L.wocr_detector_destroy(None)


def test_model_flattening_roundtrip():
    """Every node, attribute and initializer of a synthetic model reaches the C structs."""
    from wocr import synth
    m = synth.pp_rec_model(classes=10)
    h = _lib.CModelHolder(m)
    c = h.c
    assert c.n_nodes == len(m.nodes)
    assert c.n_inits == len(m.weights) + len(m.ints)
    for k, n in enumerate(m.nodes):
        cn = c.nodes[k]
        assert cn.op.decode() == n.op
        assert [cn.inputs[i].decode() for i in range(cn.n_inputs)] == n.inputs
        assert cn.n_attrs == len(n.attrs)
    names = {c.inits[i].name.decode() for i in range(c.n_inits)}
    assert names == set(m.weights) | set(m.ints)


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES", None) is None and
                    __import__("torch").cuda.is_available(), reason="a GPU is present")
def test_no_device_is_an_error_not_a_crash():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = wocr.lib().wocr_ctx_create(0, 8, ctypes.byref(h))
    assert st != 0
    assert wocr.lib().wocr_last_error()
    with pytest.raises(wocr.WocrError):
        wocr.Gpu()
