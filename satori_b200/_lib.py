"""ctypes binding of ``libsatori_cuda.so`` (the C ABI in include/satori_cuda.h).

There is no fallback: if the library is missing or cannot be loaded, every call raises.  The
library is built in-tree by ``satori_b200/build.py`` (``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libsatori_cuda.so")

OK = 0
ERR_ARGUMENT = 1
ERR_INVALID_DATA = 2
ERR_NOT_SUPPORTED = 3
ERR_CONTEXT_FULL = 4
ERR_DISPOSED = 5
ERR_CUDA = 6
ERR_TIMEOUT = 7
ERR_OUT_OF_MEMORY = 8

Q8_0, Q4_0, T2_64, T2_128, T2_256 = 0, 1, 64, 128, 256
Q4_K, Q6_K = 12, 14
TB_64, TB_128, TB_256 = 1064, 1128, 1256
ORDER_EXECUTE, ORDER_SCALAR, ORDER_BATCH, ORDER_TENSOR = 0, 1, 2, 3


class SatoriError(RuntimeError):
    """A failed C-ABI call; ``status`` is the satori_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


# One Python exception per C# exception the reference throws for the same condition.
class ArgumentError(SatoriError, ValueError):               # ArgumentException / ArgumentOutOfRangeException
    pass


class InvalidDataError(SatoriError):                        # InvalidDataException
    pass


class NotSupportedError(SatoriError, NotImplementedError):  # NotSupportedException
    pass


class ContextFullError(SatoriError):                        # InvalidOperationException (context limit)
    pass


class DisposedError(SatoriError):                           # ObjectDisposedException
    pass


class DeviceError(SatoriError, IOError):                    # device failure / bounded wait expired
    pass


_STATUS_EXC = {ERR_ARGUMENT: ArgumentError, ERR_INVALID_DATA: InvalidDataError, ERR_NOT_SUPPORTED: NotSupportedError,
               ERR_CONTEXT_FULL: ContextFullError, ERR_DISPOSED: DisposedError, ERR_CUDA: DeviceError,
               ERR_TIMEOUT: DeviceError, ERR_OUT_OF_MEMORY: DeviceError}

_lib = None
_lock = threading.Lock()

_vp = C.c_void_p
_i32p = C.POINTER(C.c_int)


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("data", _vp), ("bytes", C.c_size_t), ("format", C.c_int),
                ("rows", C.c_int), ("cols", C.c_int)]


class ModelDesc(C.Structure):
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("ffn", C.c_int), ("q_heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("rms_epsilon", C.c_float),
                ("rope_base", C.c_double), ("tied_embeddings", C.c_int), ("n_tensors", C.c_int),
                ("tensors", C.POINTER(Tensor))]


# name -> (restype, argtypes)
_SIGS = {
    "satori_init": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "satori_destroy": (C.c_int, [_vp]),
    "satori_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "satori_version": (C.c_int, [C.c_char_p, C.c_size_t]),
    "satori_stream": (_vp, [_vp]),
    "satori_set_stream": (C.c_int, [_vp, _vp]),
    "satori_synchronize": (C.c_int, [_vp]),
    "satori_matrix_create": (C.c_int, [_vp, _vp, C.c_size_t, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    "satori_matrix_create_device": (C.c_int, [_vp, _vp, C.c_size_t, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    "satori_matrix_execute": (C.c_int, [_vp, _vp, _vp]),
    "satori_matrix_execute_scalar": (C.c_int, [_vp, _vp, _vp]),
    "satori_matrix_execute_batch": (C.c_int, [_vp, _vp, C.c_int, _vp]),
    "satori_matrix_execute_tensor": (C.c_int, [_vp, _vp, C.c_int, _vp]),
    "satori_matrix_execute_device": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int]),
    "satori_matrix_read_row": (C.c_int, [_vp, C.c_int, _vp]),
    "satori_matrix_info": (C.c_int, [_vp, _i32p, _i32p, _i32p, C.POINTER(C.c_size_t)]),
    "satori_matrix_device_payload": (_vp, [_vp]),
    "satori_matrix_destroy": (C.c_int, [_vp]),
    "satori_ternary2_quantize": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, _vp]),
    "satori_quantize_q_device": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, _vp]),
    "satori_grouped_attention_device": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp]),
    "satori_grouped_attention": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp]),
    "satori_grouped_attention_noalloc": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp]),
    "satori_rope_half": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, C.c_double, C.c_int]),
    "satori_attn_create": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_double, C.POINTER(_vp)]),
    "satori_attn_append": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp]),
    "satori_attn_destroy": (C.c_int, [_vp]),
    "satori_session_create": (C.c_int, [_vp, C.POINTER(ModelDesc), C.c_int, C.POINTER(_vp)]),
    "satori_session_create_sharded": (C.c_int, [_vp, C.POINTER(ModelDesc), C.c_int, C.c_int, C.c_int, _vp,
                                                C.POINTER(_vp)]),
    "satori_nccl_unique_id": (C.c_int, [_vp]),
    "satori_matrix_create_sharded": (C.c_int, [_vp, _vp, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                              _vp, C.POINTER(_vp)]),
    "satori_matrix_sharded_execute_device": (C.c_int, [_vp, _vp, _vp, C.c_int]),
    "satori_matrix_sharded_execute": (C.c_int, [_vp, _vp, _vp, C.c_int]),
    "satori_matrix_sharded_info": (C.c_int, [_vp, _i32p, _i32p]),
    "satori_matrix_sharded_destroy": (C.c_int, [_vp]),
    "satori_session_append": (C.c_int, [_vp, C.c_int, _vp, _i32p]),
    "satori_session_append_tokens": (C.c_int, [_vp, _vp, C.c_int, _vp, _i32p]),
"satori_session_forward_tensor": (C.c_int, [_vp, _vp, C.c_int, _vp, _i32p]),
    "satori_session_generate": (C.c_int, [_vp, C.c_int, C.c_int, _vp]),
    "satori_session_position": (C.c_int, [_vp, _i32p]),
    "satori_session_reset": (C.c_int, [_vp]),
    "satori_session_rewind": (C.c_int, [_vp, C.c_int]),
    "satori_session_info": (C.c_int, [_vp, _i32p, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "satori_session_stage": (C.c_int, [_vp, C.c_int, _vp, C.c_size_t]),
    "satori_session_destroy": (C.c_int, [_vp]),
    "satori_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "satori_gguf_close": (C.c_int, [_vp]),
    "satori_gguf_counts": (C.c_int, [_vp, _i32p, _i32p]),
    "satori_gguf_tensor_info": (C.c_int, [_vp, C.c_int, C.c_char_p, C.c_size_t, _i32p, _i32p,
                                          C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "satori_gguf_find_tensor": (C.c_int, [_vp, C.c_char_p, _i32p]),
    "satori_gguf_tensor_data": (_vp, [_vp, C.c_int]),
    "satori_gguf_metadata": (C.c_int, [_vp, C.c_int, C.c_char_p, C.c_size_t, _i32p, _i32p, C.POINTER(C.c_int64)]),
    "satori_gguf_read_scalar": (C.c_int, [_vp, C.c_char_p, _i32p, _vp, C.c_size_t, C.POINTER(C.c_size_t)]),
    "satori_gguf_model_desc": (C.c_int, [_vp, C.POINTER(ModelDesc), _vp, C.c_int, _i32p]),
    "satori_session_create_from_gguf": (C.c_int, [_vp, _vp, C.c_int, C.POINTER(_vp)]),
    "satori_stq2_open": (C.c_int, [_vp, C.c_char_p, C.POINTER(_vp)]),
}

EXPORTED = tuple(_SIGS)


def header_symbols(header_path: str | None = None) -> list[str]:
    """Function names declared in include/satori_cuda.h (used by the export test)."""
    import re
    if header_path is None:
        header_path = os.path.join(os.path.dirname(_HERE), "include", "satori_cuda.h")
    text = open(header_path).read()
    return sorted(set(re.findall(r"SATORI_API\s+[\w\s\*]*?\b(satori_\w+)\s*\(", text)))


def lib() -> C.CDLL:
    """Load the library (raises if it is missing: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"{LIB_PATH} is missing; run __graft_entry__.build() or satori_b200/build.py")
                L = C.CDLL(LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().satori_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, where: str = "") -> None:
    if status != OK:
        msg = last_error()
        exc = _STATUS_EXC.get(status, SatoriError)
        raise exc(status, f"{where}: {msg}" if where else msg)


def version() -> str:
    buf = C.create_string_buffer(128)
    check(lib().satori_version(buf, len(buf)), "satori_version")
    return buf.value.decode()
