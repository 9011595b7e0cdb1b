"""A small GGUF v3 writer for the tests (this repository's own; the reference builds its test containers
with GgufContainerFixture.Prefix, tests/Satori.Numerics.Tests/GgufContainerFixture.cs:15-34, and its
fixture generator fixtures/gguf/v1/generate.py)."""
from __future__ import annotations

import struct

import numpy as np

# metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_PACK = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
         U64: "<Q", I64: "<q", F64: "<d"}
# tensor types
T_F32, T_F16, T_Q4_0, T_Q8_0, T_Q4_K, T_Q6_K = 0, 1, 2, 8, 12, 14


def gstr(s) -> bytes:
    b = s.encode("utf-8") if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def value(t: int, v) -> bytes:
    if t == STR:
        return gstr(v)
    if t == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(value(et, i) for i in items)
    return struct.pack(_PACK[t], v)


def entry(key: str, t: int, v) -> bytes:
    return gstr(key) + struct.pack("<I", t) + value(t, v)


def prefix(alignment: int, meta: bytes = b"", extras: int = 0, tensors=None, arch: str = "llama",
           tensor_count=None) -> bytes:
    """Header + catalogue, padded to `alignment` (GgufContainerFixture.Prefix): general.architecture and
    general.alignment, then `extras` caller entries in `meta`, then tensors (name, dims, type, offset)."""
    if tensors is None:
        tensors = [("first", [2], 0, 0), ("second", [2], 1, alignment)]
    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors) if tensor_count is None else tensor_count, 2 + extras))
    out += entry("general.architecture", STR, arch) + entry("general.alignment", U32, alignment) + meta
    for name, dims, t, off in tensors:
        out += gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", t, off)
    while len(out) % alignment:
        out += b"\0"
    return bytes(out)


def file_with(prefix_bytes: bytes, total: int) -> bytes:
    """The prefix followed by zeros up to `total` bytes (MappedFileFixture)."""
    return prefix_bytes + b"\0" * max(0, total - len(prefix_bytes))


def model_gguf(spec, tensors: dict, alignment: int = 32, arch: str = "qwen2", extra_meta=()) -> bytes:
    """A qwen2-style model container holding `tensors` (payload bytes or float32 vectors) in canonical
    order, with the metadata DenseTransformerAdapter reads."""
    kv = [("general.architecture", STR, arch), ("general.alignment", U32, alignment),
          ("general.quantization_version", U32, 2),
          (f"{arch}.block_count", U32, spec.layers), (f"{arch}.embedding_length", U32, spec.hidden),
          (f"{arch}.feed_forward_length", U32, spec.ffn), (f"{arch}.attention.head_count", U32, spec.q_heads),
          (f"{arch}.attention.head_count_kv", U32, spec.kv_heads),
          (f"{arch}.attention.layer_norm_rms_epsilon", F32, spec.eps), (f"{arch}.rope.freq_base", F32, spec.rope_base)]
    kv += list(extra_meta)
    shapes = spec.matrix_shapes()
    body = bytearray()
    cat = bytearray()
    off = 0
    blobs = []
    for name, data in tensors.items():
        arr = np.ascontiguousarray(data)
        if name in shapes:
            rows, cols = shapes[name]
            dims = [cols, rows]
            t = T_Q8_0 if spec.format_of(name) == 0 else T_Q4_0
            raw = arr.astype(np.uint8).tobytes()
        else:
            dims = [arr.size]
            t = T_F32
            raw = arr.astype(np.float32).tobytes()
        cat += gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        cat += struct.pack("<IQ", t, off)
        pad = (-len(raw)) % alignment
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)))
    for k, t, v in kv:
        head += entry(k, t, v)
    head += cat
    while len(head) % alignment:
        head += b"\0"
    return bytes(head) + b"".join(blobs)
