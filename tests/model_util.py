"""Seeded synthetic Qwen2-style models for the session tests (host tensors, oracle quantizer).

Weights are N(0, 0.02^2) as in BASELINE configs 4-5; norm weights are 1 + N(0, 0.1^2) and biases
N(0, 0.02^2).  The quantizer is this repository's own (the reference only decodes GGUF), so the
same payload bytes feed both the GPU session and the oracle session.
"""
from __future__ import annotations

import numpy as np


def synthetic_tensors(spec, seed: int = 1234) -> dict:
    from oracle import oracle
    rng = np.random.default_rng(seed)
    tensors = {}
    for name, (rows, cols) in spec.matrix_shapes().items():
        w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
        tensors[name] = oracle.q_quantize(w, rows, cols, spec.format_of(name))
        del w
    for name, n in spec.vector_shapes().items():
        if name.endswith("norm.weight"):
            tensors[name] = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        else:
            tensors[name] = (0.02 * rng.standard_normal(n)).astype(np.float32)
    return tensors
