"""Host-side mirror of Satori's MatVec and attention API over the CUDA C ABI.

Names, argument meaning and error behaviour follow the C# reference so that a caller (or a
test) reads the same:

* ``QuantizedMatrixShape`` / ``BlockQuantization``     -- src/Satori.Core/QuantizedMatrixShape.cs:5-22
* ``CudaMatrixFactory.create``                         -- IQuantizedMatrixFactory.Create (IQuantizedMatrixFactory.cs:6)
* ``CudaQuantizedMatrix.execute``                      -- IQuantizedMatrix.Execute (IQuantizedMatrix.cs:6)
* ``Ternary2Matrix`` / ``Ternary2MatVec``              -- src/Satori.Core/Ternary2Matrix.cs, Ternary2MatVec.cs
* ``MappedTernary2Matrix``                             -- src/Satori.Core/MappedTernary2Matrix.cs
* ``TransformerOps.grouped_attention`` / ``rope_half`` -- src/Satori.Core/TransformerOps.cs:99-179

All arithmetic runs on the GPU through ``libsatori_cuda.so``; this module only moves bytes.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
import struct
import threading

import numpy as np

from . import _lib
from ._lib import ArgumentError, DisposedError, InvalidDataError, check

_vp = C.c_void_p


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _f32(a, n: int | None = None, name: str = "vector") -> np.ndarray:
    v = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    if n is not None and v.size != n:
        raise ArgumentError(_lib.ERR_ARGUMENT, f"{name} length {v.size} does not match {n}")
    return v


def _u8(a) -> np.ndarray:
    if isinstance(a, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(a), dtype=np.uint8)
    return np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)


def _commit(y: np.ndarray, output):
    """Output is written only after the device call succeeded (IQuantizedMatrix.cs:6)."""
    if output is None:
        return y
    if output.dtype != np.float32 or output.size != y.size:
        raise ArgumentError(_lib.ERR_ARGUMENT, "output length does not match")
    output.reshape(-1)[:] = y
    return output


# --------------------------------------------------------------------------- context
class Context:
    """One CUDA device and stream (one per caller thread, like VulkanContext)."""

    def __init__(self, device: int = 0):
        h = _vp()
        check(_lib.lib().satori_init(device, C.byref(h)), "satori_init")
        self._h = h
        self.device = device

    @property
    def handle(self):
        if not self._h:
            raise DisposedError(_lib.ERR_DISPOSED, "context is disposed")
        return self._h

    @property
    def stream(self) -> int:
        return _lib.lib().satori_stream(self.handle) or 0

    def set_stream(self, stream_ptr: int | None) -> None:
        """Route device work to a caller-owned cudaStream_t (None restores the context's own)."""
        check(_lib.lib().satori_set_stream(self.handle, stream_ptr), "set_stream")

    def synchronize(self) -> None:
        check(_lib.lib().satori_synchronize(self.handle), "satori_synchronize")

    def close(self) -> None:
        if self._h:
            _lib.lib().satori_destroy(self._h)
            self._h = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


_default_contexts: dict[int, Context] = {}
_default_lock = threading.Lock()


def default_context(device: int = 0) -> Context:
    with _default_lock:
        ctx = _default_contexts.get(device)
        if ctx is None:
            ctx = _default_contexts[device] = Context(device)
        return ctx


# --------------------------------------------------------------------------- shapes
class BlockQuantization(enum.IntEnum):
    """src/Satori.Core/BlockQuantization.cs:3 (values are the GGUF tensor type ids of the K formats)."""
    Q8_0 = _lib.Q8_0
    Q4_0 = _lib.Q4_0
    Q4_K = _lib.Q4_K
    Q6_K = _lib.Q6_K


_BLOCKS = {BlockQuantization.Q8_0: (32, 34), BlockQuantization.Q4_0: (32, 18), BlockQuantization.Q4_K: (256, 144),
           BlockQuantization.Q6_K: (256, 210)}


class QuantizedMatrixShape:
    """QuantizedMatrixShape (QuantizedMatrixShape.cs:5-22): positive dims, complete blocks per row (32 weights
    for Q8_0 / Q4_0, 256 for the K super-blocks)."""

    def __init__(self, rows: int, columns: int, fmt: BlockQuantization):
        fmt = BlockQuantization(fmt)
        self.block_elements, self.block_bytes = _BLOCKS[fmt]
        if rows <= 0 or columns <= 0 or columns % self.block_elements != 0:
            raise ArgumentError(_lib.ERR_ARGUMENT,
                                f"Positive dimensions and complete {self.block_elements}-weight rows required.")
        self.rows, self.columns, self.format = rows, columns, fmt
        self.byte_length = rows * (columns // self.block_elements) * self.block_bytes
        if self.byte_length > 0x7FFFFFFF:
            raise ArgumentError(_lib.ERR_ARGUMENT, "payload exceeds Int32 limits")

    def __repr__(self):
        return f"QuantizedMatrixShape({self.rows}, {self.columns}, {self.format.name})"


def ternary2_byte_length(rows: int, columns: int, block_size: int) -> int:
    """Ternary2Shape.ByteLength (Ternary2Shape.cs:14)."""
    if rows <= 0 or columns <= 0:
        raise ArgumentError(_lib.ERR_ARGUMENT, "dimensions must be positive")
    if block_size not in (64, 128, 256):
        raise ArgumentError(_lib.ERR_ARGUMENT, "Supported block sizes: 64, 128, 256.")
    n = rows * ((columns + block_size - 1) // block_size) * (4 + block_size // 4)
    if n > 0x7FFFFFFF:
        raise ArgumentError(_lib.ERR_ARGUMENT, "payload exceeds Int32 limits")
    return n


# --------------------------------------------------------------------------- resident matrices
class CudaQuantizedMatrix:
    """A resident payload on the device (IQuantizedMatrix).  Q8_0/Q4_0 or Ternary2."""

    def __init__(self, ctx: Context, payload, rows: int, columns: int, fmt: int):
        self.ctx = ctx
        h = _vp()
        data = _u8(payload)
        check(_lib.lib().satori_matrix_create(ctx.handle, _ptr(data), data.size, rows, columns, fmt, C.byref(h)),
              "create")
        self._h = h
        self.rows, self.columns, self.format = rows, columns, fmt

    @classmethod
    def from_device(cls, ctx: Context, device_ptr: int, nbytes: int, rows: int, columns: int, fmt: int):
        m = cls.__new__(cls)
        m.ctx = ctx
        h = _vp()
        check(_lib.lib().satori_matrix_create_device(ctx.handle, device_ptr, nbytes, rows, columns, fmt, C.byref(h)),
              "create_device")
        m._h = h
        m.rows, m.columns, m.format = rows, columns, fmt
        return m

    @classmethod
    def _adopt(cls, ctx: Context, handle):
        """Wraps a matrix handle created by a native loader (satori_stq2_open)."""
        m = cls.__new__(cls)
        m.ctx = ctx
        m._h = handle
        rows, cols, fmt, nbytes = C.c_int(), C.c_int(), C.c_int(), C.c_size_t()
        check(_lib.lib().satori_matrix_info(handle, C.byref(rows), C.byref(cols), C.byref(fmt), C.byref(nbytes)),
              "info")
        m.rows, m.columns, m.format = rows.value, cols.value, fmt.value
        return m

    @property
    def handle(self):
        if not self._h:
            raise DisposedError(_lib.ERR_DISPOSED, "matrix is disposed")
        return self._h

    def execute(self, input, output: np.ndarray | None = None) -> np.ndarray:
        """IQuantizedMatrix.Execute: output is written only when the call succeeds."""
        x = _f32(input, self.columns, "input")
        y = np.empty(self.rows, np.float32)
        check(_lib.lib().satori_matrix_execute(self.handle, _ptr(x), _ptr(y)), "execute")
        return _commit(y, output)

    def execute_scalar(self, input, output: np.ndarray | None = None) -> np.ndarray:
        x = _f32(input, self.columns, "input")
        y = np.empty(self.rows, np.float32)
        check(_lib.lib().satori_matrix_execute_scalar(self.handle, _ptr(x), _ptr(y)), "execute_scalar")
        return _commit(y, output)

    def execute_batch(self, input, positions: int, output: np.ndarray | None = None, threads: int = 1) -> np.ndarray:
        """QuantizedMatVec.ExecuteBatch (position-major); `threads` is accepted for signature parity."""
        if positions <= 0 or threads <= 0:
            raise ArgumentError(_lib.ERR_ARGUMENT, "positions and threads must be positive")
        x = _f32(input, positions * self.columns, "input")
        y = np.empty(positions * self.rows, np.float32)
        check(_lib.lib().satori_matrix_execute_batch(self.handle, _ptr(x), positions, _ptr(y)), "execute_batch")
        return _commit(y, output)

    def execute_tensor(self, input, positions: int, output: np.ndarray | None = None) -> np.ndarray:
        """ExecuteBatch's product on the tensor cores (Q8_0 / Q4_0): exact products, FP32 accumulation in
        tensor memory -- not the reference's operation order, within a few FP32 roundings of it."""
        if positions <= 0:
            raise ArgumentError(_lib.ERR_ARGUMENT, "positions must be positive")
        x = _f32(input, positions * self.columns, "input")
        y = np.empty(positions * self.rows, np.float32)
        check(_lib.lib().satori_matrix_execute_tensor(self.handle, _ptr(x), positions, _ptr(y)), "execute_tensor")
        return _commit(y, output)

    def execute_device(self, dx: int, dy: int, positions: int = 1, order: int = _lib.ORDER_BATCH) -> None:
        check(_lib.lib().satori_matrix_execute_device(self.handle, dx, dy, positions, order), "execute_device")

    def read_row(self, row: int) -> np.ndarray:
        """GgufQuantizedMatrix.ReadRow (bit-exact decode; Q4_0 rejected as in the reference)."""
        out = np.empty(self.columns, np.float32)
        check(_lib.lib().satori_matrix_read_row(self.handle, row, _ptr(out)), "read_row")
        return out

    @property
    def device_payload(self) -> int:
        return _lib.lib().satori_matrix_device_payload(self.handle) or 0

    def dispose(self) -> None:
        if self._h:
            _lib.lib().satori_matrix_destroy(self._h)
            self._h = _vp()

    close = dispose

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass


def sharded_matrix_rows(rows: int, rank: int, world: int) -> tuple:
    """Rows [begin, end) that rank `rank` of `world` holds in a row-sharded matrix (the rule of
    satori_matrix_create_sharded): blocks of S = ceil(rows / world) rows, the last one shorter; every rank
    must receive at least one row."""
    if world < 1 or not 0 <= rank < world or rows <= 0:
        raise ArgumentError(_lib.ERR_ARGUMENT, f"bad rank {rank} / world {world} / rows {rows}")
    s = -(-rows // world)
    if s * (world - 1) >= rows:
        raise _lib.NotSupportedError(_lib.ERR_NOT_SUPPORTED, f"{rows} rows leave rank {world - 1} of {world} without rows")
    return rank * s, min(rows, (rank + 1) * s)


class CudaShardedMatrix:
    """One large MatVec split by rows over the GPUs of a node (one process per GPU): rank r holds rows
    [r*S, min((r+1)*S, rows)), S = ceil(rows / world), computes them with the single-GPU kernels (each row
    bit-exact in the requested order) and NCCL all-gathers the full output onto every rank.  Every rank
    passes the WHOLE payload (only its rows are uploaded) and the same NCCL id; execute is a collective."""

    def __init__(self, ctx: Context, payload, shape: QuantizedMatrixShape, rank: int, world: int, nccl_id: bytes):
        self.ctx = ctx
        self.rows, self.columns, self.format = shape.rows, shape.columns, int(shape.format)
        h = _vp()
        if hasattr(payload, "data_ptr"):
            ptr, nbytes, on_dev = int(payload.data_ptr()), int(payload.numel() * payload.element_size()), 1
            keep = None
        else:
            keep = _u8(payload)
            ptr, nbytes, on_dev = keep.ctypes.data, keep.nbytes, 0
        idbuf = C.create_string_buffer(bytes(nccl_id), 128) if nccl_id is not None else None
        check(_lib.lib().satori_matrix_create_sharded(ctx.handle, ptr, nbytes, self.rows, self.columns, self.format,
                                                      on_dev, rank, world, idbuf, C.byref(h)), "create_sharded")
        del keep
        self._h = h
        b, e = C.c_int(), C.c_int()
        check(_lib.lib().satori_matrix_sharded_info(h, C.byref(b), C.byref(e)), "sharded_info")
        self.row_begin, self.row_end = b.value, e.value

    @property
    def handle(self):
        if self._h is None or not self._h.value:
            raise DisposedError(_lib.ERR_DISPOSED, "matrix is disposed")
        return self._h

    def execute(self, input, order: int = _lib.ORDER_BATCH, output: np.ndarray | None = None) -> np.ndarray:
        x = _f32(input, self.columns, "input")
        y = np.empty(self.rows, np.float32)
        check(_lib.lib().satori_matrix_sharded_execute(self.handle, _ptr(x), _ptr(y), order), "sharded_execute")
        return _commit(y, output)

    def execute_device(self, dx: int, dy: int, order: int = _lib.ORDER_BATCH) -> None:
        check(_lib.lib().satori_matrix_sharded_execute_device(self.handle, dx, dy, order), "sharded_execute_device")

    def dispose(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.lib().satori_matrix_sharded_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass


class CudaMatrixFactory:
    """IQuantizedMatrixFactory over the GPU (the seam VulkanContext implements in the reference)."""

    def __init__(self, ctx: Context | None = None):
        self.ctx = ctx or default_context()

    def create(self, payload, shape: QuantizedMatrixShape) -> CudaQuantizedMatrix:
        data = _u8(payload)
        if data.size != shape.byte_length:
            raise ArgumentError(_lib.ERR_ARGUMENT, "Incorrect quantized payload length.")
        return CudaQuantizedMatrix(self.ctx, data, shape.rows, shape.columns, int(shape.format))


# --------------------------------------------------------------------------- Ternary2
_STQ2_HEADER = 32


class Ternary2Matrix:
    """Validated row-major ternary weights with FP32 block scales (Ternary2Matrix.cs)."""

    def __init__(self, rows: int, columns: int, block_size: int, data: np.ndarray, ctx: Context | None = None,
                 _validated_device: CudaQuantizedMatrix | None = None):
        self.rows, self.columns, self.block_size = rows, columns, block_size
        self._data = data
        self._ctx = ctx or default_context()
        self._dev = _validated_device

    @property
    def byte_length(self) -> int:
        return self._data.size

    @property
    def data(self) -> np.ndarray:
        return self._data

    def copy_data_to(self, destination: np.ndarray) -> None:
        destination.reshape(-1)[: self._data.size] = self._data

    @property
    def device(self) -> CudaQuantizedMatrix:
        if self._dev is None:
            self._dev = CudaQuantizedMatrix(self._ctx, self._data, self.rows, self.columns, self.block_size)
        return self._dev

    @staticmethod
    def quantize(weights, rows: int, columns: int, block_size: int = 64, ctx: Context | None = None) -> "Ternary2Matrix":
        """Ternary2Matrix.Quantize (Ternary2Matrix.cs:38-71), computed on the device, bit-exact."""
        ctx = ctx or default_context()
        n = ternary2_byte_length(rows, columns, block_size)
        w = np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
        if w.size != rows * columns:
            raise ArgumentError(_lib.ERR_ARGUMENT, "Weights must match matrix dimensions.")
        out = np.zeros(n, np.uint8)
        check(_lib.lib().satori_ternary2_quantize(ctx.handle, _ptr(w), rows, columns, block_size, _ptr(out)), "quantize")
        return Ternary2Matrix(rows, columns, block_size, out, ctx)

    @staticmethod
    def from_packed(rows: int, columns: int, block_size: int, data, ctx: Context | None = None) -> "Ternary2Matrix":
        """Ternary2Matrix.FromPacked (:73-81): length and payload validated (ArgumentError)."""
        ctx = ctx or default_context()
        owned = _u8(data).copy()
        if owned.size != ternary2_byte_length(rows, columns, block_size):
            raise ArgumentError(_lib.ERR_ARGUMENT, "Payload length must match matrix dimensions.")
        dev = CudaQuantizedMatrix(ctx, owned, rows, columns, block_size)
        return Ternary2Matrix(rows, columns, block_size, owned, ctx, dev)

    def dequantize(self, destination: np.ndarray | None = None) -> np.ndarray:
        """Ternary2Matrix.Dequantize (:103-120), decoded on the device row by row."""
        out = np.empty((self.rows, self.columns), np.float32)
        for r in range(self.rows):
            out[r] = self.device.read_row(r)
        return _commit(out.reshape(-1), destination)

    def save(self, path: str) -> None:
        """Ternary2Matrix.Save (:29-36): STQ2 header then the payload; refuses to overwrite."""
        with open(path, "xb") as fh:
            fh.write(stq2_header(self.rows, self.columns, self.block_size))
            fh.write(self._data.tobytes())


# --------------------------------------------------------------------------- ternary bitplane (STB1)
_TB_FORMAT = {64: _lib.TB_64, 128: _lib.TB_128, 256: _lib.TB_256}


class TernaryBitplaneMatrix:
    """Ternary weights in the bitplane layout (TernaryBitplaneMatrix.cs, docs/ternary-bitplane-v1.md): the
    same blocks and scales as Ternary2 with a positive and a negative bit plane per block."""

    def __init__(self, rows: int, columns: int, block_size: int, data: np.ndarray, device: CudaQuantizedMatrix):
        self.rows, self.columns, self.block_size = rows, columns, block_size
        self._data = data
        self.device = device

    @property
    def byte_length(self) -> int:
        return self._data.size

    @property
    def data(self) -> np.ndarray:
        return self._data

    def copy_data_to(self, destination: np.ndarray) -> None:
        destination.reshape(-1)[: self._data.size] = self._data

    @staticmethod
    def from_packed(rows: int, columns: int, block_size: int, payload, ctx: Context | None = None):
        """TernaryBitplaneMatrix.FromPacked (:57-64): length, scales, planes and padding validated on the
        device (ArgumentError, like the reference's ArgumentException)."""
        ctx = ctx or default_context()
        owned = _u8(payload).copy()
        if owned.size != ternary2_byte_length(rows, columns, block_size):
            raise ArgumentError(_lib.ERR_ARGUMENT, "Incorrect bitplane payload length.")
        dev = CudaQuantizedMatrix(ctx, owned, rows, columns, _TB_FORMAT[block_size])
        return TernaryBitplaneMatrix(rows, columns, block_size, owned, dev)

    @staticmethod
    def from_ternary2(matrix: "Ternary2Matrix") -> "TernaryBitplaneMatrix":
        """TernaryBitplaneMatrix.FromTernary2 (:18-36): scale bytes copied, code 1 -> P bit, code 2 -> N bit."""
        bs, bb = matrix.block_size, 4 + matrix.block_size // 4
        src = matrix.data.reshape(-1, bb)
        codes = np.stack([(src[:, 4:] >> (2 * k)) & 3 for k in range(4)], axis=2).reshape(src.shape[0], bs)
        out = np.zeros_like(src)
        out[:, :4] = src[:, :4]
        out[:, 4:4 + bs // 8] = np.packbits(codes == 1, axis=1, bitorder="little")
        out[:, 4 + bs // 8:] = np.packbits(codes == 2, axis=1, bitorder="little")
        return TernaryBitplaneMatrix.from_packed(matrix.rows, matrix.columns, bs, out.reshape(-1), matrix._ctx)

    def to_ternary2(self) -> "Ternary2Matrix":
        """TernaryBitplaneMatrix.ToTernary2 (:38-55): P -> 01, N -> 10, byte-identical to the original."""
        bs, bb = self.block_size, 4 + self.block_size // 4
        src = self._data.reshape(-1, bb)
        p = np.unpackbits(src[:, 4:4 + bs // 8], axis=1, bitorder="little").astype(np.uint8)
        n = np.unpackbits(src[:, 4 + bs // 8:], axis=1, bitorder="little").astype(np.uint8)
        codes = (p | (n << 1)).reshape(src.shape[0], bs // 4, 4)
        out = np.zeros_like(src)
        out[:, :4] = src[:, :4]
        out[:, 4:] = codes[:, :, 0] | (codes[:, :, 1] << 2) | (codes[:, :, 2] << 4) | (codes[:, :, 3] << 6)
        return Ternary2Matrix.from_packed(self.rows, self.columns, bs, out.reshape(-1), self.device.ctx)

    def save(self, path: str) -> None:
        """TernaryBitplaneMatrix.Save (:89-97): the STB1 header then the payload; refuses to overwrite."""
        with open(path, "xb") as fh:
            fh.write(b"STB1" + stq2_header(self.rows, self.columns, self.block_size)[4:])
            fh.write(self._data.tobytes())

    @staticmethod
    def load(path: str, ctx: Context | None = None) -> "TernaryBitplaneMatrix":
        """TernaryBitplaneMatrix.Load (:99-117) with TernaryBitplaneFileFormat.ReadHeader: any defect of the
        header, length or payload is an InvalidDataError."""
        raw = open(path, "rb").read()
        if len(raw) < _STQ2_HEADER or raw[:4] != b"STB1":
            raise InvalidDataError(_lib.ERR_INVALID_DATA, "Invalid bitplane file.")
        rows, cols, bs = stq2_read_header(b"STQ2" + raw[4:32])
        if len(raw) != _STQ2_HEADER + ternary2_byte_length(rows, cols, bs):
            raise InvalidDataError(_lib.ERR_INVALID_DATA, "Incorrect bitplane file length.")
        try:
            return TernaryBitplaneMatrix.from_packed(rows, cols, bs, np.frombuffer(raw[32:], np.uint8), ctx)
        except ArgumentError as e:
            raise InvalidDataError(_lib.ERR_INVALID_DATA, "Invalid bitplane file.") from e


class TernaryBitplaneMatVec:
    """TernaryBitplaneMatVec (TernaryBitplaneMatVec.cs): Execute runs the AVX2-order arithmetic."""

    @staticmethod
    def execute(matrix: TernaryBitplaneMatrix, input, output: np.ndarray | None = None) -> np.ndarray:
        _check_t2_vectors(matrix.rows, matrix.columns, input, output)
        return matrix.device.execute(input, output)

    execute_avx2 = execute

    @staticmethod
    def execute_scalar(matrix: TernaryBitplaneMatrix, input, output: np.ndarray | None = None) -> np.ndarray:
        _check_t2_vectors(matrix.rows, matrix.columns, input, output)
        return matrix.device.execute_scalar(input, output)


def stq2_header(rows: int, columns: int, block_size: int) -> bytes:
    """Ternary2FileFormat.WriteHeader (Ternary2FileFormat.cs:9-19)."""
    n = ternary2_byte_length(rows, columns, block_size)
    return b"STQ2" + struct.pack("<HHiiiiq", 1, _STQ2_HEADER, rows, columns, block_size, 0, n)


def stq2_read_header(header: bytes) -> tuple[int, int, int]:
    """Ternary2FileFormat.ReadHeader (Ternary2FileFormat.cs:21-35); InvalidDataError on any mismatch."""
    if len(header) < _STQ2_HEADER or header[:4] != b"STQ2":
        raise InvalidDataError(_lib.ERR_INVALID_DATA, "Unsupported Ternary2 header.")
    version, size, rows, cols, bs, pad, length = struct.unpack("<HHiiiiq", header[4:32])
    if version != 1 or size != _STQ2_HEADER or pad != 0:
        raise InvalidDataError(_lib.ERR_INVALID_DATA, "Unsupported Ternary2 header.")
    try:
        want = ternary2_byte_length(rows, cols, bs)
    except ArgumentError as e:
        raise InvalidDataError(_lib.ERR_INVALID_DATA, "Invalid Ternary2 shape or payload.") from e
    if length != want:
        raise InvalidDataError(_lib.ERR_INVALID_DATA, "Payload length disagrees with matrix shape.")
    return rows, cols, bs


def _check_t2_vectors(rows, cols, input, output):
    """Ternary2MatVec.ValidateVectors (Ternary2MatVec.cs:30-36)."""
    n_in = np.asarray(input).size
    n_out = rows if output is None else np.asarray(output).size
    if n_in != cols or n_out != rows:
        raise ArgumentError(_lib.ERR_ARGUMENT, "Vector lengths must match matrix dimensions.")
    if output is not None and isinstance(input, np.ndarray) and np.shares_memory(input, output):
        raise ArgumentError(_lib.ERR_ARGUMENT, "Output must not overlap input.")


class Ternary2MatVec:
    """Ternary2MatVec (Ternary2MatVec.cs:7-50): Execute runs the AVX2-order arithmetic on the GPU."""

    @staticmethod
    def execute(matrix: Ternary2Matrix, input, output: np.ndarray | None = None) -> np.ndarray:
        _check_t2_vectors(matrix.rows, matrix.columns, input, output)
        return matrix.device.execute(input, output)

    execute_avx2 = execute

    @staticmethod
    def execute_scalar(matrix: Ternary2Matrix, input, output: np.ndarray | None = None) -> np.ndarray:
        _check_t2_vectors(matrix.rows, matrix.columns, input, output)
        return matrix.device.execute_scalar(input, output)


class MappedTernary2Matrix:
    """A validated STQ2 file executed on the GPU (MappedTernary2Matrix.cs:9-55).

    The payload is read once from the mapped file and uploaded unchanged; every invalid header,
    length or payload raises InvalidDataError, as the reference's constructor does (:25-28).
    """

    def __init__(self, path: str, ctx: Context | None = None):
        ctx = ctx or default_context()
        size = os.path.getsize(path)
        mm = np.memmap(path, dtype=np.uint8, mode="r") if size else np.zeros(0, np.uint8)
        if mm.size < _STQ2_HEADER:
            raise InvalidDataError(_lib.ERR_INVALID_DATA, "Truncated Ternary2 header.")
        rows, cols, bs = stq2_read_header(bytes(mm[:_STQ2_HEADER]))
        n = ternary2_byte_length(rows, cols, bs)
        if mm.size != _STQ2_HEADER + n:
            raise InvalidDataError(_lib.ERR_INVALID_DATA, "Truncated payload or trailing file data.")
        try:
            self._dev = CudaQuantizedMatrix(ctx, np.ascontiguousarray(mm[_STQ2_HEADER:]), rows, cols, bs)
        except ArgumentError as e:
            raise InvalidDataError(_lib.ERR_INVALID_DATA, "Invalid Ternary2 shape or payload.") from e
        del mm
        self.rows, self.columns, self.block_size, self.byte_length = rows, cols, bs, n
        self._disposed = False

    def _live(self) -> CudaQuantizedMatrix:
        if self._disposed:
            raise DisposedError(_lib.ERR_DISPOSED, "Cannot access a disposed object.")
        return self._dev

    def execute(self, input, output: np.ndarray | None = None) -> np.ndarray:
        dev = self._live()
        _check_t2_vectors(self.rows, self.columns, input, output)
        return dev.execute(input, output)

    def execute_scalar(self, input, output: np.ndarray | None = None) -> np.ndarray:
        dev = self._live()
        _check_t2_vectors(self.rows, self.columns, input, output)
        return dev.execute_scalar(input, output)

    def dispose(self) -> None:
        if not self._disposed:
            self._dev.dispose()
            self._disposed = True

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


# --------------------------------------------------------------------------- attention
class TransformerOps:
    """GPU restatements of the attention operators (TransformerOps.cs)."""

    @staticmethod
    def grouped_attention(query, keys, values, query_heads: int, kv_heads: int, head_dimension: int,
                          token_count: int, output: np.ndarray | None = None, ctx: Context | None = None) -> np.ndarray:
        """TransformerOps.GroupedAttention (:140-179)."""
        ctx = ctx or default_context()
        if head_dimension <= 0 or query_heads <= 0 or kv_heads <= 0 or query_heads % kv_heads or token_count <= 0:
            raise ArgumentError(_lib.ERR_ARGUMENT, "Invalid grouped-attention dimensions.")
        q = _f32(query, query_heads * head_dimension, "query")
        k = _f32(keys, token_count * kv_heads * head_dimension, "keys")
        v = _f32(values, token_count * kv_heads * head_dimension, "values")
        out = np.empty(q.size, np.float32)
        check(_lib.lib().satori_grouped_attention(ctx.handle, _ptr(q), _ptr(k), _ptr(v), query_heads, kv_heads,
                                                  head_dimension, token_count, _ptr(out)), "grouped_attention")
        return _commit(out, output)

    @staticmethod
    def attention(query, keys, values, head_dimension: int, token_count: int, output=None, ctx=None) -> np.ndarray:
        """TransformerOps.Attention (:62-94): equal query and KV heads."""
        q = _f32(query)
        if head_dimension <= 0 or q.size == 0 or q.size % head_dimension:
            raise ArgumentError(_lib.ERR_ARGUMENT, "Invalid attention dimensions.")
        heads = q.size // head_dimension
        return TransformerOps.grouped_attention(q, keys, values, heads, heads, head_dimension, token_count, output, ctx)

    @staticmethod
    def rope_half(vector: np.ndarray, head_dimension: int, position: int, frequency_base: float,
                  rotary_dimensions: int, ctx: Context | None = None) -> np.ndarray:
        """TransformerOps.RopeHalf (:99-118), in place on a float32 array."""
        ctx = ctx or default_context()
        if vector.dtype != np.float32 or not vector.flags.c_contiguous:
            raise ArgumentError(_lib.ERR_ARGUMENT, "vector must be a contiguous float32 array")
        check(_lib.lib().satori_rope_half(ctx.handle, _ptr(vector), vector.size, head_dimension, position,
                                          float(frequency_base), rotary_dimensions), "rope_half")
        return vector


class AttentionCache:
    """Device KV cache plus the attention half of DenseForward.Step (DenseForward.cs:135-143)."""

    def __init__(self, layers: int, context: int, q_heads: int, kv_heads: int, head_dim: int, rope_base: float,
                 ctx: Context | None = None):
        self.ctx = ctx or default_context()
        h = _vp()
        check(_lib.lib().satori_attn_create(self.ctx.handle, layers, context, q_heads, kv_heads, head_dim,
                                            float(rope_base), C.byref(h)), "attn_create")
        self._h = h
        self.q_width, self.kv_width = q_heads * head_dim, kv_heads * head_dim

    def append(self, layer: int, position: int, q, k, v) -> np.ndarray:
        if not self._h:
            raise DisposedError(_lib.ERR_DISPOSED, "attention cache is disposed")
        qv, kv, vv = _f32(q, self.q_width, "q"), _f32(k, self.kv_width, "k"), _f32(v, self.kv_width, "v")
        out = np.empty(self.q_width, np.float32)
        check(_lib.lib().satori_attn_append(self._h, layer, position, _ptr(qv), _ptr(kv), _ptr(vv), _ptr(out)), "append")
        return out

    def dispose(self):
        if self._h:
            _lib.lib().satori_attn_destroy(self._h)
            self._h = _vp()

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass
