"""satori_b200 -- the Satori decode hot path (quantized MatVec + decode attention) on B200.

The compute lives in ``_build/libsatori_cuda.so`` (hand-written sm_100a CUDA behind the C ABI in
``include/satori_cuda.h``); this package mirrors the reference's C# API over that ABI.
"""
from ._lib import (ArgumentError, ContextFullError, DeviceError, DisposedError, InvalidDataError,
                   NotSupportedError, SatoriError, ORDER_BATCH, ORDER_EXECUTE, ORDER_SCALAR, Q4_0, Q8_0, Q4_K, Q6_K,
                   T2_64, T2_128, T2_256, version)
from .core import (AttentionCache, BlockQuantization, Context, CudaMatrixFactory, CudaQuantizedMatrix, CudaShardedMatrix,
                   MappedTernary2Matrix, QuantizedMatrixShape, Ternary2Matrix, Ternary2MatVec, TernaryBitplaneMatrix,
                   TernaryBitplaneMatVec, TransformerOps,
                   default_context, sharded_matrix_rows, stq2_header, stq2_read_header, ternary2_byte_length)
from .gguf import GgufFile, GgufMetadata, GgufTensor, open_stq2, session_from_gguf
from .model import (CudaDenseSession, ModelSpec, broadcast_nccl_id, nccl_unique_id, qwen2_1_5b, qwen2_7b,
                    shard_ranges, tiny)

__all__ = [
    "ArgumentError", "ContextFullError", "DeviceError", "DisposedError", "InvalidDataError", "NotSupportedError",
    "SatoriError", "ORDER_BATCH", "ORDER_EXECUTE", "ORDER_SCALAR", "Q4_0", "Q8_0", "Q4_K", "Q6_K", "T2_64", "T2_128", "T2_256",
    "version", "AttentionCache", "BlockQuantization", "Context", "CudaMatrixFactory", "CudaQuantizedMatrix",
    "CudaShardedMatrix",
    "MappedTernary2Matrix", "QuantizedMatrixShape", "Ternary2Matrix", "Ternary2MatVec", "TernaryBitplaneMatrix",
    "TernaryBitplaneMatVec", "TransformerOps",
    "default_context", "sharded_matrix_rows", "stq2_header", "stq2_read_header", "ternary2_byte_length", "CudaDenseSession", "ModelSpec",
    "qwen2_1_5b", "qwen2_7b", "tiny", "nccl_unique_id", "broadcast_nccl_id", "shard_ranges",
    "GgufFile", "GgufMetadata", "GgufTensor", "open_stq2", "session_from_gguf",
]
