"""wocr: the inference hot path of huppiflupp/wgpu-ocr on B200 (sm_100a CUDA behind a C ABI).

Public API (mirrors the reference crate): `Gpu`, `Detector`, `Recognizer`, `NdGraph`, the PP-OCRv6
page pipeline `PPPipeline`, plus the host-side greedy CTC decoders.  Model descriptions are `wocr.model.Model`; seeded synthetic
models and inputs of the benchmark configurations are in `wocr.synth`.
"""
from ._lib import EXPORTS, LIB_PATH, WocrError, lib
from .api import (Batch, Detector, Gpu, NdGraph, OcrsPipeline, Pending, PPPipeline, Recognizer, load_pp_dictionary,
                  ocrs_decode, pad_line, pp_decode, text_lines)
from .model import Model, Node
from .onnx import load_onnx, parse_onnx

__all__ = ["Gpu", "Batch", "Pending", "Detector", "Recognizer", "NdGraph", "PPPipeline", "OcrsPipeline", "text_lines", "pad_line", "WocrError", "Model", "Node", "ocrs_decode",
           "pp_decode", "load_pp_dictionary", "lib", "LIB_PATH", "EXPORTS", "load_onnx", "parse_onnx"]
