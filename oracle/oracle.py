"""ctypes/numpy wrapper over the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs import this module,
and only as the checker.  The product path (``satori_b200``) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

OK, ERR_ARGUMENT, ERR_INVALID_DATA, ERR_NOT_SUPPORTED, ERR_CONTEXT_FULL = 0, 1, 2, 3, 4
Q8_0, Q4_0 = 0, 1

_lib = None
_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)
_f64p = C.POINTER(C.c_double)
_i32p = C.POINTER(C.c_int)


class OracleError(RuntimeError):
    def __init__(self, code: int, where: str):
        super().__init__(f"{where}: oracle status {code}")
        self.code = code


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = _build.LIB_PATH
        if not os.path.exists(path) and os.path.exists(os.path.join(_build.HERE, "satori_oracle.c")):
            _build.build_oracle()
        _lib = C.CDLL(path)
        L = _lib
        L.so_half_to_float.restype = C.c_float
        L.so_half_to_float.argtypes = [C.c_uint16]
        L.so_float_to_half.restype = C.c_uint16
        L.so_float_to_half.argtypes = [C.c_float]
        L.so_session_create.restype = C.c_void_p
        L.so_session_create.argtypes = [C.c_void_p, C.c_int]
        L.so_session_destroy.argtypes = [C.c_void_p]
        L.so_session_reset.argtypes = [C.c_void_p]
        L.so_session_fill_cache.argtypes = [C.c_void_p, C.c_int, C.c_uint32]
        L.so_session_position.argtypes = [C.c_void_p]
        L.so_session_append.argtypes = [C.c_void_p, C.c_int, _f32p, _i32p, C.c_int]
        L.so_session_stage.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_int]
    return _lib


def _u8(a: np.ndarray):
    return a.ctypes.data_as(_u8p)


def _f32(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _check(code: int, where: str):
    if code != OK:
        raise OracleError(code, where)


def _c_u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(a), dtype=np.uint8) if isinstance(a, (bytes, bytearray))
                                else a, dtype=np.uint8)


def _c_f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- helpers
def half_to_float(bits: int) -> float:
    return lib().so_half_to_float(bits)


def float_to_half(value: float) -> int:
    return lib().so_float_to_half(value)


# ---------------------------------------------------------------- Ternary2
def t2_geometry(rows: int, cols: int, bs: int):
    bpr, bb, ln = C.c_int(), C.c_int(), C.c_int64()
    _check(lib().so_t2_geometry(rows, cols, bs, C.byref(bpr), C.byref(bb), C.byref(ln)), "t2_geometry")
    return bpr.value, bb.value, ln.value


def t2_quantize(w: np.ndarray, rows: int, cols: int, bs: int = 64) -> np.ndarray:
    _, _, ln = t2_geometry(rows, cols, bs)
    w = _c_f32(w).reshape(-1)
    if w.size != rows * cols:
        raise OracleError(ERR_ARGUMENT, "t2_quantize")
    out = np.zeros(ln, dtype=np.uint8)
    _check(lib().so_t2_quantize(_f32(w), rows, cols, bs, _u8(out)), "t2_quantize")
    return out


def t2_validate(data, rows: int, cols: int, bs: int) -> int:
    d = _c_u8(data)
    return lib().so_t2_validate(_u8(d), C.c_int64(d.size), rows, cols, bs)


def t2_dequantize(data, rows: int, cols: int, bs: int) -> np.ndarray:
    d = _c_u8(data)
    out = np.zeros(rows * cols, dtype=np.float32)
    _check(lib().so_t2_dequantize(_u8(d), rows, cols, bs, _f32(out)), "t2_dequantize")
    return out


def t2_matvec(data, rows: int, cols: int, bs: int, x, order: str = "avx2", threads: int = 1) -> np.ndarray:
    d, xv = _c_u8(data), _c_f32(x)
    y = np.zeros(rows, dtype=np.float32)
    L = lib()
    if order == "avx2":
        rc = L.so_t2_matvec_avx2(_u8(d), rows, cols, bs, _f32(xv), _f32(y), threads)
    elif order == "avx2_emulated":
        rc = L.so_t2_matvec_avx2_emulated(_u8(d), rows, cols, bs, _f32(xv), _f32(y))
    elif order == "scalar":
        rc = L.so_t2_matvec_scalar(_u8(d), rows, cols, bs, _f32(xv), _f32(y))
    else:
        raise ValueError(order)
    _check(rc, "t2_matvec")
    return y


def stq2_header(rows: int, cols: int, bs: int) -> bytes:
    h = (C.c_uint8 * 32)()
    lib().so_stq2_write_header(h, rows, cols, bs)
    return bytes(h)


def stq2_read_header(data: bytes):
    d = _c_u8(data)
    r, c, b = C.c_int(), C.c_int(), C.c_int()
    rc = lib().so_stq2_read_header(_u8(d), C.c_int64(d.size), C.byref(r), C.byref(c), C.byref(b))
    _check(rc, "stq2_read_header")
    return r.value, c.value, b.value


# ---------------------------------------------------------------- Q8_0 / Q4_0
def q_geometry(rows: int, cols: int, fmt: int):
    bb, ln = C.c_int(), C.c_int64()
    _check(lib().so_q_geometry(rows, cols, fmt, C.byref(bb), C.byref(ln)), "q_geometry")
    return bb.value, ln.value


def q_validate(data, rows: int, cols: int, fmt: int) -> int:
    d = _c_u8(data)
    return lib().so_q_validate(_u8(d), C.c_int64(d.size), rows, cols, fmt)


def q_decode_row(row_bytes, cols: int, fmt: int) -> np.ndarray:
    d = _c_u8(row_bytes)
    out = np.zeros(cols, dtype=np.float32)
    _check(lib().so_q_decode_row(_u8(d), cols, fmt, _f32(out)), "q_decode_row")
    return out


def q_matvec(data, rows: int, cols: int, fmt: int, x, order: str = "batch", positions: int = 1,
             threads: int = 1) -> np.ndarray:
    d, xv = _c_u8(data), _c_f32(x)
    L = lib()
    if order == "batch":
        y = np.zeros(rows * positions, dtype=np.float32)
        rc = L.so_q_matvec_batch(_u8(d), rows, cols, fmt, _f32(xv), positions, _f32(y), threads)
    elif order == "batch_emulated":
        y = np.zeros(rows * positions, dtype=np.float32)
        rc = L.so_q_matvec_batch_emulated(_u8(d), rows, cols, fmt, _f32(xv), positions, _f32(y))
    elif order == "avx2":
        y = np.zeros(rows, dtype=np.float32)
        rc = L.so_q_matvec_avx2(_u8(d), rows, cols, fmt, _f32(xv), _f32(y), threads)
    elif order == "avx2_emulated":
        y = np.zeros(rows, dtype=np.float32)
        rc = L.so_q_matvec_avx2_emulated(_u8(d), rows, cols, fmt, _f32(xv), _f32(y))
    elif order == "scalar":
        y = np.zeros(rows, dtype=np.float32)
        rc = L.so_q_matvec_scalar(_u8(d), rows, cols, fmt, _f32(xv), _f32(y))
    else:
        raise ValueError(order)
    _check(rc, "q_matvec")
    return y


def q_quantize(w: np.ndarray, rows: int, cols: int, fmt: int) -> np.ndarray:
    _, ln = q_geometry(rows, cols, fmt)
    w = _c_f32(w).reshape(-1)
    out = np.zeros(ln, dtype=np.uint8)
    _check(lib().so_q_quantize(_f32(w), rows, cols, fmt, _u8(out)), "q_quantize")
    return out


# ---------------------------------------------------------------- K-quants (Q4_K, Q6_K; Q8_K activations)
Q4_K, Q6_K = 12, 14


def k_geometry(rows: int, cols: int, fmt: int):
    bb, ln = C.c_int(), C.c_int64()
    _check(lib().so_k_geometry(rows, cols, fmt, C.byref(bb), C.byref(ln)), "k_geometry")
    return bb.value, ln.value


def k_validate(data, rows: int, cols: int, fmt: int) -> int:
    d = _c_u8(data)
    return lib().so_k_validate(_u8(d), C.c_int64(d.size), rows, cols, fmt)


def k_decode_row(row_bytes, cols: int, fmt: int) -> np.ndarray:
    d = _c_u8(row_bytes)
    out = np.zeros(cols, dtype=np.float32)
    _check(lib().so_k_decode_row(_u8(d), cols, fmt, _f32(out)), "k_decode_row")
    return out


def k_matvec(data, rows: int, cols: int, fmt: int, x, order: str = "batch", positions: int = 1,
             threads: int = 1) -> np.ndarray:
    d, xv = _c_u8(data), _c_f32(x)
    L = lib()
    if order == "batch":
        y = np.zeros(rows * positions, dtype=np.float32)
        rc = L.so_k_matvec_batch(_u8(d), rows, cols, fmt, _f32(xv), positions, _f32(y), threads)
    elif order == "avx2":
        y = np.zeros(rows, dtype=np.float32)
        rc = L.so_k_matvec_avx2(_u8(d), rows, cols, fmt, _f32(xv), _f32(y), threads)
    elif order == "scalar":
        y = np.zeros(rows, dtype=np.float32)
        rc = L.so_k_matvec_scalar(_u8(d), rows, cols, fmt, _f32(xv), _f32(y))
    else:
        raise ValueError(order)
    _check(rc, "k_matvec")
    return y


def q8k_quantize_row(x) -> np.ndarray:
    xv = _c_f32(x)
    out = np.zeros(xv.size // 256 * 292, dtype=np.uint8)
    _check(lib().so_q8k_quantize_row(_f32(xv), xv.size, _u8(out)), "q8k_quantize_row")
    return out


def k_int_dot(block, fmt: int, activation):
    """(integer product, min product) of one K-quant block with one Q8_K activation block."""
    b, a = _c_u8(block), _c_u8(activation)
    dot, mins = C.c_int32(), C.c_int32()
    _check(lib().so_k_int_dot(_u8(b), fmt, _u8(a), C.byref(dot), C.byref(mins)), "k_int_dot")
    return dot.value, mins.value


# ---------------------------------------------------------------- ternary bitplane (STB1)
def tb_from_t2(t2, rows: int, cols: int, bs: int) -> np.ndarray:
    _, _, ln = t2_geometry(rows, cols, bs)
    d = _c_u8(t2)
    out = np.zeros(ln, dtype=np.uint8)
    _check(lib().so_tb_from_t2(_u8(d), rows, cols, bs, _u8(out)), "tb_from_t2")
    return out


def tb_to_t2(tb, rows: int, cols: int, bs: int) -> np.ndarray:
    _, _, ln = t2_geometry(rows, cols, bs)
    d = _c_u8(tb)
    out = np.zeros(ln, dtype=np.uint8)
    _check(lib().so_tb_to_t2(_u8(d), rows, cols, bs, _u8(out)), "tb_to_t2")
    return out


def tb_validate(data, rows: int, cols: int, bs: int) -> int:
    d = _c_u8(data)
    return lib().so_tb_validate(_u8(d), C.c_int64(d.size), rows, cols, bs)


def tb_matvec(data, rows: int, cols: int, bs: int, x, order: str = "avx2") -> np.ndarray:
    d, xv = _c_u8(data), _c_f32(x)
    y = np.zeros(rows, dtype=np.float32)
    fn = lib().so_tb_matvec_avx2 if order == "avx2" else lib().so_tb_matvec_scalar
    _check(fn(_u8(d), rows, cols, bs, _f32(xv), _f32(y)), "tb_matvec")
    return y


# ---------------------------------------------------------------- operators
def rmsnorm(x, w, eps: float) -> np.ndarray:
    xv, wv = _c_f32(x), _c_f32(w)
    out = np.zeros_like(xv)
    _check(lib().so_rmsnorm(_f32(xv), _f32(wv), xv.size, C.c_float(eps), _f32(out)), "rmsnorm")
    return out


def rmsnorm_heads(v, w, eps: float, head_dim: int) -> np.ndarray:
    vv, wv = _c_f32(v).copy(), _c_f32(w)
    _check(lib().so_rmsnorm_heads(_f32(vv), vv.size, _f32(wv), C.c_float(eps), head_dim), "rmsnorm_heads")
    return vv


def rope_half(v, head_dim: int, position: int, base: float, rotary: int) -> np.ndarray:
    vv = _c_f32(v).copy()
    _check(lib().so_rope_half(_f32(vv), vv.size, head_dim, position, C.c_double(base), rotary), "rope_half")
    return vv


def rope_interleaved(v, head_dim: int, position: int) -> np.ndarray:
    vv = _c_f32(v).copy()
    _check(lib().so_rope_interleaved(_f32(vv), vv.size, head_dim, position), "rope")
    return vv


def swiglu(gate, up) -> np.ndarray:
    g, u = _c_f32(gate), _c_f32(up)
    out = np.zeros_like(g)
    _check(lib().so_swiglu(_f32(g), _f32(u), g.size, _f32(out)), "swiglu")
    return out


def add(a, b) -> np.ndarray:
    av, bv = _c_f32(a), _c_f32(b)
    out = np.zeros_like(av)
    _check(lib().so_add(_f32(av), _f32(bv), av.size, _f32(out)), "add")
    return out


def grouped_attention(q, keys, values, q_heads: int, kv_heads: int, head_dim: int, tokens: int,
                      threads: int = 1) -> np.ndarray:
    qv, kv, vv = _c_f32(q), _c_f32(keys), _c_f32(values)
    out = np.zeros(q_heads * head_dim, dtype=np.float32)
    scores = np.zeros(max(tokens, 1), dtype=np.float64)
    rc = lib().so_grouped_attention(_f32(qv), _f32(kv), _f32(vv), q_heads, kv_heads, head_dim, tokens,
                                    scores.ctypes.data_as(_f64p), _f32(out), threads)
    _check(rc, "grouped_attention")
    return out


def greedy_select(logits) -> int:
    lv = _c_f32(logits)
    tok = C.c_int()
    _check(lib().so_greedy_select(_f32(lv), lv.size, C.byref(tok)), "greedy_select")
    return tok.value


# ---------------------------------------------------------------- dense session
class _Layer(C.Structure):
    _fields_ = [("attn_norm", _f32p), ("ffn_norm", _f32p),
                ("q_bias", _f32p), ("k_bias", _f32p), ("v_bias", _f32p),
                ("q", _u8p), ("k", _u8p), ("v", _u8p), ("o", _u8p),
                ("gate", _u8p), ("up", _u8p), ("down", _u8p),
                ("q_fmt", C.c_int), ("k_fmt", C.c_int), ("v_fmt", C.c_int), ("o_fmt", C.c_int),
                ("gate_fmt", C.c_int), ("up_fmt", C.c_int), ("down_fmt", C.c_int)]


class _Model(C.Structure):
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("ffn", C.c_int), ("q_heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int),
                ("eps", C.c_float), ("rope_base", C.c_double),
                ("embd", _u8p), ("embd_fmt", C.c_int), ("output", _u8p), ("output_fmt", C.c_int),
                ("output_norm", _f32p), ("layer", C.POINTER(_Layer))]


class OracleSession:
    """Oracle twin of ``DenseSession`` over a ``satori_b200`` model description (same tensors)."""

    def __init__(self, spec, tensors: dict, context: int):
        self._keep = []

        def u8(name):
            a = _c_u8(tensors[name])
            self._keep.append(a)
            return _u8(a)

        def f32(name):
            if name not in tensors:
                return None
            a = _c_f32(tensors[name])
            self._keep.append(a)
            return _f32(a)

        fmt = spec.format_of
        layers = (_Layer * spec.layers)()
        for i in range(spec.layers):
            p = f"blk.{i}."
            L = layers[i]
            L.attn_norm, L.ffn_norm = f32(p + "attn_norm.weight"), f32(p + "ffn_norm.weight")
            L.q_bias, L.k_bias, L.v_bias = f32(p + "attn_q.bias"), f32(p + "attn_k.bias"), f32(p + "attn_v.bias")
            for field, tname in (("q", "attn_q"), ("k", "attn_k"), ("v", "attn_v"), ("o", "attn_output"),
                                 ("gate", "ffn_gate"), ("up", "ffn_up"), ("down", "ffn_down")):
                setattr(L, field, u8(p + tname + ".weight"))
                setattr(L, field + "_fmt", fmt(p + tname + ".weight"))
        self._layers = layers
        m = _Model()
        m.layers, m.hidden, m.ffn = spec.layers, spec.hidden, spec.ffn
        m.q_heads, m.kv_heads, m.head_dim, m.vocab = spec.q_heads, spec.kv_heads, spec.head_dim, spec.vocab
        m.eps, m.rope_base = spec.eps, spec.rope_base
        m.embd, m.embd_fmt = u8("token_embd.weight"), fmt("token_embd.weight")
        m.output, m.output_fmt = u8("output.weight"), fmt("output.weight")
        m.output_norm = f32("output_norm.weight")
        m.layer = C.cast(layers, C.POINTER(_Layer))
        self._model = m
        self.vocab, self.hidden = spec.vocab, spec.hidden
        self._s = lib().so_session_create(C.byref(m), context)
        if not self._s:
            raise OracleError(ERR_ARGUMENT, "session_create")

    def append(self, token: int, threads: int = 1):
        logits = np.zeros(self.vocab, dtype=np.float32)
        arg = C.c_int()
        _check(lib().so_session_append(self._s, token, _f32(logits), C.byref(arg), threads), "session_append")
        return logits, arg.value

    def stage(self, which: int) -> np.ndarray:
        out = np.zeros(self.hidden, dtype=np.float32)
        _check(lib().so_session_stage(self._s, which, _f32(out), self.hidden), "session_stage")
        return out

    @property
    def position(self) -> int:
        return lib().so_session_position(self._s)

    def reset(self):
        lib().so_session_reset(self._s)

    def fill_cache(self, position: int, seed: int = 1):
        """Benchmark helper: seeded cache rows [0, position) and position = `position`."""
        _check(lib().so_session_fill_cache(self._s, int(position), int(seed)), "session_fill_cache")

    def close(self):
        if self._s:
            lib().so_session_destroy(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
