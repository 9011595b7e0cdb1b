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


def device_synthetic_tensors(ctx, spec, seed: int = 31) -> dict:
    """The same kind of model generated on the GPU (seeded N(0, 0.02^2) weights quantized by this
    library's device quantizer), returned as host arrays: fast enough for the 1.5B and 7B shapes."""
    import torch

    from satori_b200 import _lib
    tensors = {}
    for i, (name, (rows, cols)) in enumerate(spec.matrix_shapes().items()):
        fmt = spec.format_of(name)
        g = torch.Generator(device="cuda").manual_seed(seed + i)
        w = torch.randn(rows * cols, generator=g, device="cuda", dtype=torch.float32) * 0.02
        out = torch.empty(rows * (cols // 32) * (34 if fmt == 0 else 18), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        _lib.check(_lib.lib().satori_quantize_q_device(ctx.handle, w.data_ptr(), rows, cols, fmt, out.data_ptr()),
                   "quantize")
        ctx.synchronize()
        tensors[name] = out.cpu().numpy()
        del w, out
    rng = np.random.default_rng(seed)
    for name, n in spec.vector_shapes().items():
        if name.endswith("norm.weight"):
            tensors[name] = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        else:
            tensors[name] = (0.02 * rng.standard_normal(n)).astype(np.float32)
    torch.cuda.empty_cache()
    return tensors
