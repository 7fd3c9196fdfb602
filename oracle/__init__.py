"""CPU oracle of the wgpu-ocr hot path: test infrastructure only (see oracle/ref.py)."""
