"""GGUF and STQ2 files through the native reader: the ``GgufFile`` / ``GgufModelLoader`` /
``MappedTernary2Matrix`` mirror.

* ``GgufFile``            -- src/Satori.Formats.Gguf/GgufFile.cs:9-176 (catalogue, ``ReadScalar``,
                             ``ReadTensor``), parsed and validated by ``satori_gguf_open``;
* ``GgufFile.model_spec`` -- ModelConfig + DenseTransformerAdapter.Validate
                             (src/Satori.Core/Model/DenseTransformerAdapter.cs:12-121);
* ``session_from_gguf``   -- a ``CudaDenseSession`` whose tensors are uploaded straight from the mapping;
* ``open_stq2``           -- MappedTernary2Matrix(path) (src/Satori.Core/MappedTernary2Matrix.cs:9-30).

Parsing needs no GPU; uploads do.
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import DisposedError, check

_vp = C.c_void_p

# GGUF metadata value types (GgufFile.SkipScalar, GgufFile.cs:186-197).
UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64, FLOAT64 = range(13)
_FMT = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i", FLOAT32: "<f",
        UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}


@dataclass(frozen=True)
class GgufTensor:
    """GgufTensor (src/Satori.Formats.Gguf/GgufTensor.cs): dimensions fastest first."""
    name: str
    dimensions: tuple
    type: int
    offset: int
    byte_length: int


@dataclass(frozen=True)
class GgufMetadata:
    key: str
    type: int
    element_type: int | None
    element_count: int


class GgufFile:
    """A validated GGUF v3 catalogue over a read-only mapping (closed by ``close`` / ``with``)."""

    def __init__(self, path: str):
        h = _vp()
        check(_lib.lib().satori_gguf_open(str(path).encode(), C.byref(h)), "GgufFile")
        self._h = h
        L = _lib.lib()
        nt, nm = C.c_int(), C.c_int()
        check(L.satori_gguf_counts(h, C.byref(nt), C.byref(nm)), "counts")
        self.tensors: dict[str, GgufTensor] = {}
        name = C.create_string_buffer(256)
        for i in range(nt.value):
            typ, rank = C.c_int(), C.c_int()
            dims = (C.c_int64 * 4)()
            off, nbytes = C.c_int64(), C.c_int64()
            check(L.satori_gguf_tensor_info(h, i, name, 256, C.byref(typ), C.byref(rank), dims, C.byref(off),
                                            C.byref(nbytes)), "tensor_info")
            n = name.value.decode()
            self.tensors[n] = GgufTensor(n, tuple(dims[d] for d in range(rank.value)), typ.value, off.value, nbytes.value)
        self.metadata: dict[str, GgufMetadata] = {}
        key = C.create_string_buffer(65536)
        for i in range(nm.value):
            typ, et, cnt = C.c_int(), C.c_int(), C.c_int64()
            check(L.satori_gguf_metadata(h, i, key, 65536, C.byref(typ), C.byref(et), C.byref(cnt)), "metadata")
            k = key.value.decode()
            self.metadata[k] = GgufMetadata(k, typ.value, et.value if typ.value == ARRAY else None,
                                            cnt.value if typ.value == ARRAY else 1)

    @property
    def handle(self):
        if not self._h:
            raise DisposedError(_lib.ERR_DISPOSED, "GGUF file is closed")
        return self._h

    def read_scalar(self, key: str):
        """GgufFile.ReadScalar: the value of a scalar entry (strings as str, booleans as bool)."""
        n, typ = C.c_size_t(), C.c_int()
        check(_lib.lib().satori_gguf_read_scalar(self.handle, key.encode(), C.byref(typ), None, 0, C.byref(n)),
              "read_scalar")
        buf = C.create_string_buffer(max(1, n.value))
        check(_lib.lib().satori_gguf_read_scalar(self.handle, key.encode(), C.byref(typ), buf, n.value, C.byref(n)),
              "read_scalar")
        raw = buf.raw[:n.value]
        if typ.value == STRING:
            return raw.decode("utf-8")
        if typ.value == BOOL:
            return raw[0] != 0
        return struct.unpack(_FMT[typ.value], raw)[0]

    def read_tensor(self, name: str, offset: int = 0, length: int | None = None) -> np.ndarray:
        """GgufFile.ReadTensor (src/Satori.Formats.Gguf/GgufFile.cs:42-48): a copy of the window
        [offset, offset + length) of the tensor's payload, the rest of the payload when ``length`` is None.
        A window outside the payload raises ArgumentError (ArgumentOutOfRangeException) before the
        mapping is touched; a closed file raises DisposedError."""
        t = self.tensors[name]
        if length is None:
            length = t.byte_length - offset
        if offset < 0 or length < 0 or offset > t.byte_length or length > t.byte_length - offset:
            raise _lib.ArgumentError(_lib.ERR_ARGUMENT, "Window exceeds tensor payload.")
        idx = C.c_int()
        check(_lib.lib().satori_gguf_find_tensor(self.handle, name.encode(), C.byref(idx)), "find_tensor")
        ptr = _lib.lib().satori_gguf_tensor_data(self.handle, idx.value)
        return np.frombuffer(C.string_at(ptr + offset, length), dtype=np.uint8).copy()

    def model_desc(self) -> dict:
        """DenseTransformerAdapter.Validate: the model shape the file describes."""
        d = _lib.ModelDesc()
        needed = C.c_int()
        check(_lib.lib().satori_gguf_model_desc(self.handle, C.byref(d), None, 0, C.byref(needed)), "model_desc")
        return {"layers": d.layers, "hidden": d.hidden, "ffn": d.ffn, "q_heads": d.q_heads, "kv_heads": d.kv_heads,
                "head_dim": d.head_dim, "vocab": d.vocab, "rms_epsilon": d.rms_epsilon, "rope_base": d.rope_base,
                "tied_embeddings": bool(d.tied_embeddings), "tensors": needed.value}

    def close(self) -> None:
        if self._h:
            _lib.lib().satori_gguf_close(self._h)
            self._h = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def session_from_gguf(path: str, context_length: int, ctx=None):
    """A CudaDenseSession over a qwen2/qwen3 GGUF file (every tensor uploaded once from the mapping)."""
    from .core import default_context
    from .model import CudaDenseSession
    ctx = ctx or default_context()
    with GgufFile(path) as g:
        h = _vp()
        check(_lib.lib().satori_session_create_from_gguf(ctx.handle, g.handle, int(context_length), C.byref(h)),
              "session_create_from_gguf")
        shape = g.model_desc()
    return CudaDenseSession._adopt(h, ctx, context_length, shape)


def open_stq2(path: str, ctx=None):
    """MappedTernary2Matrix(path): a validated STQ2 file as a resident CudaQuantizedMatrix."""
    from .core import CudaQuantizedMatrix, default_context
    ctx = ctx or default_context()
    h = _vp()
    check(_lib.lib().satori_stq2_open(ctx.handle, str(path).encode(), C.byref(h)), "stq2_open")
    return CudaQuantizedMatrix._adopt(ctx, h)
