"""wocr: the inference hot path of huppiflupp/wgpu-ocr on B200 (sm_100a CUDA behind a C ABI).

Public API (mirrors the reference crate): `Gpu`, `Detector`, `Recognizer`, `NdGraph`, plus the
host-side greedy CTC decoders.  Model descriptions are `wocr.model.Model`; seeded synthetic
models and inputs of the benchmark configurations are in `wocr.synth`.
"""
from ._lib import EXPORTS, LIB_PATH, WocrError, lib
from .api import Detector, Gpu, NdGraph, Recognizer, ocrs_decode, pp_decode
from .model import Model, Node
from .onnx import load_onnx, parse_onnx

__all__ = ["Gpu", "Detector", "Recognizer", "NdGraph", "WocrError", "Model", "Node", "ocrs_decode", "pp_decode",
           "lib", "LIB_PATH", "EXPORTS", "load_onnx", "parse_onnx"]
