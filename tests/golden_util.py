"""Deterministic corpora the reference's tests use, restated for this suite.

* ``numerical_random`` / ``critical_cases`` -- NumericalCorpus.cs:8-47 (Xorshift32, seed 1729,
  ``(s >> 8) / 2^23 - 1`` in FP32) and its CriticalCases list (:18-29).
* ``q8_critical_cases`` / ``q8_input`` -- Q8Validation.CriticalCases / Input (Q8Validation.cs:9-28).
* ``attention_boundary_inputs`` -- the formulas of tools/attention_reference.py:4-6.
* ``gamma_bound`` -- the FP64 error bound of NumericalValidation.cs:23-46 and Q8Validation.cs:30-53.
"""
from __future__ import annotations

import json
import math
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_fixtures.json")
_golden_cache = None

FLT_MAX = float(np.finfo(np.float32).max)
FLT_EPS_DENORM = float(np.float32(1.401298464324817e-45))  # C# float.Epsilon (smallest subnormal)
HALF_EPSILON = 5.960464477539063e-08                        # C# Half.Epsilon as float


def golden() -> dict:
    global _golden_cache
    if _golden_cache is None:
        with open(GOLDEN) as fh:
            _golden_cache = json.load(fh)
    return _golden_cache


class Xorshift32:
    def __init__(self, seed: int = 1729):
        self.state = seed & 0xFFFFFFFF

    def next(self) -> np.float32:
        s = self.state
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        self.state = s
        return np.float32(np.float32(s >> 8) * np.float32(1.0 / 8388608.0)) - np.float32(1.0)


def numerical_random(rows: int, cols: int):
    """NumericalCorpus.RandomMatrix: weights = Next()*2, then the input."""
    rng = Xorshift32()
    w = np.array([np.float32(rng.next() * np.float32(2)) for _ in range(rows * cols)], dtype=np.float32)
    x = np.array([rng.next() for _ in range(cols)], dtype=np.float32)
    return "random", rows, cols, w, x


def _pattern(name, rows, cols, weight, activation):
    w = np.array([weight(i) for i in range(rows * cols)], dtype=np.float32)
    x = np.array([activation(i) for i in range(cols)], dtype=np.float32)
    return name, rows, cols, w, x


def critical_cases(bs: int):
    yield numerical_random(7, bs * 2 + 3)
    yield _pattern("zeros", 3, bs + 1, lambda i: 0.0, lambda i: 1.0)
    yield _pattern("alternating", 5, bs * 2 + 1, lambda i: 1.0 if i % 2 == 0 else -1.0, lambda i: 1.0)
    yield _pattern("sparse", 3, bs - 1, lambda i: 4.0 if i % 17 == 0 else 0.0, lambda i: float(i % 3 - 1))
    yield _pattern("small-scale", 3, bs + 3, lambda i: 1e-30 if i % 2 == 0 else -1e-30, lambda i: 1.0)
    yield _pattern("large-scale", 3, bs + 3, lambda i: 1e30 if i % 2 == 0 else -1e30, lambda i: 1e-10)
    yield _pattern("subnormal", 2, bs + 1, lambda i: FLT_EPS_DENORM if i % 2 == 0 else -FLT_EPS_DENORM, lambda i: 1.0)
    yield _pattern("max-scale", 2, bs + 1, lambda i: FLT_MAX if i % 2 == 0 else -FLT_MAX, lambda i: 1e-38)
    yield _pattern("single-weight", 1, 1, lambda i: -2.0, lambda i: 3.0)


def t2_bound_ok(payload: np.ndarray, rows: int, cols: int, bs: int, x: np.ndarray, y: np.ndarray) -> bool:
    """NumericalValidation.Evaluate's bound (NumericalValidation.cs:23-46) on dequantized weights."""
    from oracle import oracle
    recon = oracle.t2_dequantize(payload, rows, cols, bs).astype(np.float64).reshape(rows, cols)
    blocks = (cols + bs - 1) // bs
    ops = bs + blocks + 2
    eps = 2.0 ** -24
    gamma = ops * eps / (1 - ops * eps)
    terms = recon * x.astype(np.float64)[None, :]
    exact = terms.sum(axis=1)
    mag = np.abs(terms).sum(axis=1)
    bound = gamma * mag + (cols + blocks) * FLT_EPS_DENORM
    err = np.abs(y.astype(np.float64) - exact)
    return bool(np.all(np.isfinite(y)) and np.all(err <= bound))


def q8_input(cols: int) -> np.ndarray:
    return np.array([((i * 17 % 31) - 15) / 16.0 for i in range(cols)], dtype=np.float32)


def q8_critical_cases():
    from oracle import oracle
    scales = [0.5, -2.0, 0.0, -0.0, HALF_EPSILON, 65504.0, 1.0]
    for rows in (1, 7, 63, 64, 65, 129):
        for cols in (32, 64, 96, 288, 768):
            bpr = cols // 32
            payload = np.zeros(rows * bpr * 34, dtype=np.uint8)
            for r in range(rows):
                for b in range(bpr):
                    off = (r * bpr + b) * 34
                    h = oracle.float_to_half(scales[(r + b) % len(scales)])
                    payload[off] = h & 0xFF
                    payload[off + 1] = h >> 8
                    for j in range(32):
                        payload[off + 2 + j] = ((r * 32 + b * 17 + j * 7) % 256 - 128) & 0xFF
            yield f"signed-scales-{rows}x{cols}", rows, cols, payload, q8_input(cols)


def q_reference_fp64(payload: np.ndarray, rows: int, cols: int, fmt: int, x: np.ndarray):
    """Independent FP64 decode-and-dot (Q8Validation.Compare, Q8Validation.cs:30-53)."""
    bb = 34 if fmt == 0 else 18
    bpr = cols // 32
    p = payload.reshape(rows, bpr, bb)
    d = p[:, :, 0:2].copy().view(np.float16).astype(np.float64).reshape(rows, bpr)
    if fmt == 0:
        q = p[:, :, 2:].view(np.int8).astype(np.float64)
    else:
        qb = p[:, :, 2:].astype(np.int32)
        q = np.concatenate([(qb & 15) - 8, (qb >> 4) - 8], axis=2).astype(np.float64)
    prod = d[:, :, None] * q * x.astype(np.float64).reshape(bpr, 32)[None, :, :]
    return prod.reshape(rows, cols).sum(axis=1), np.abs(prod).reshape(rows, cols).sum(axis=1)


def gamma_bound(cols: int, magnitude: np.ndarray) -> np.ndarray:
    n = cols + cols / 32.0 + 2
    gamma = n * 2.0 ** -24 / (1 - n * 2.0 ** -24)
    return gamma * magnitude + n * FLT_EPS_DENORM


def attention_boundary_inputs():
    """tools/attention_reference.py:4-6: width 288 = 6 heads x 48, 128 tokens."""
    width = 288
    f32 = np.float32
    q = np.array([f32((i % 17 - 8) * .125) for i in range(width)], dtype=np.float32)
    k = np.array([[f32(((t * 13 + i * 7) % 31 - 15) * .0625) for i in range(width)] for t in range(128)],
                 dtype=np.float32)
    v = np.array([[f32(((t * 5 + i * 11) % 37 - 18) * .125) for i in range(width)] for t in range(128)],
                 dtype=np.float32)
    return q, k, v


def operator_close(actual, expected, abs_tol=2e-6, rel_tol=2e-6) -> bool:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return bool(a.shape == e.shape and np.all(np.isfinite(a)) and np.all(np.abs(a - e) <= abs_tol + rel_tol * np.abs(e)))


def north_star_close(actual, expected, rel=1e-5, abs_=1e-6):
    """The north_star tolerance: |a - e| <= 1e-5 * |e| + 1e-6."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return np.abs(a - e) <= rel * np.abs(e) + abs_


def bits_equal(a, b) -> bool:
    """Bit-exact FP32 equality, treating +0 and -0 as equal (their values are equal)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    if a.shape != b.shape:
        return False
    same = a.view(np.uint32) == b.view(np.uint32)
    zero = (a == 0) & (b == 0)
    return bool(np.all(same | zero))


def seeded_normal(seed: int, n: int, sigma: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(n) * sigma).astype(np.float32)


def isclose_rel(a: float, b: float, tol: float) -> bool:
    return math.isclose(a, b, rel_tol=tol, abs_tol=tol)
