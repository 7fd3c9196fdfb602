"""The model description handed to the executors: an ONNX graph after loading.

This mirrors the data the reference's loader produces (`src/onnx.rs:44-56`, `Onnx::load`
`src/onnx.rs:88-123`): a node list in graph order (op type, input and output value names,
attributes), float initializers with their dimensions, integer (int64) constants, the graph's
input name (the first input that is not an initializer) and its output name (the first graph
output). `Constant` nodes are already turned into initializers or integer lists, as the
reference's loader does.

The C ABI (`include/wocr.h`, `wocr_model`) takes exactly this description; `wocr._lib` flattens
a `Model` into those structs.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Union

import numpy as np

AttrValue = Union[int, float, str, List[int], List[float]]


@dataclass
class Node:
    """One ONNX node (`src/onnx.rs:16-42`)."""

    op: str
    inputs: List[str]
    outputs: List[str]
    attrs: Dict[str, AttrValue] = field(default_factory=dict)

    def ints(self, name):
        v = self.attrs.get(name)
        return None if v is None else [int(x) for x in v]

    def int(self, name):
        v = self.attrs.get(name)
        return None if v is None else int(v)

    def string(self, name):
        v = self.attrs.get(name)
        return None if v is None else str(v)

    def attr_f32(self, name):
        v = self.attrs.get(name)
        return None if v is None else float(v)


@dataclass
class Model:
    """`Onnx` of `src/onnx.rs:44-56`: nodes, float weights, integer constants, input, output."""

    nodes: List[Node]
    weights: Dict[str, np.ndarray]
    ints: Dict[str, np.ndarray]
    input: str
    output: str

    def weight(self, name: str) -> np.ndarray:
        if name not in self.weights:
            raise KeyError(f"missing weight {name}")
        return self.weights[name]

    def readers(self, name: str) -> int:
        """How many nodes read `name` (`src/onnx.rs:129-132`)."""
        return sum(1 for n in self.nodes if name in n.inputs)

    def param_count(self) -> int:
        return int(sum(w.size for w in self.weights.values()))
