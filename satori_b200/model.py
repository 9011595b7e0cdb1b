"""Dense decode session on the GPU: the ``IInferenceSession`` / ``DenseSession`` mirror.

``ModelSpec`` carries the ``ModelShape`` fields (src/Satori.Core/Model/ModelShape.cs:10-24) plus the
tensor formats; tensors are named as in GGUF (``token_embd.weight``, ``blk.N.attn_q.weight`` ...,
DenseForward.cs:308-330).  ``CudaDenseSession`` uploads every tensor once and runs
``DenseSession.Append`` (DenseSession.cs:111-131) -- embed, every layer's ``DenseForward.Step``, the
final norm and logits, greedy argmax -- as one captured CUDA graph per token.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import ArgumentError, DisposedError, NotSupportedError, check
from .core import Context, default_context

_vp = C.c_void_p


@dataclass
class ModelSpec:
    layers: int
    hidden: int
    ffn: int
    q_heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    eps: float = 1e-6
    rope_base: float = 1e6
    tied_embeddings: bool = False
    has_bias: bool = True
    proj_format: int = _lib.Q8_0          # all projections
    embd_format: int = _lib.Q8_0          # token_embd.weight (Q8_0: Q4_0 rows are unsupported)
    output_format: int = _lib.Q8_0        # output.weight
    name: str = "custom"
    formats: dict = field(default_factory=dict)

    @property
    def q_width(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim

    def format_of(self, name: str) -> int:
        if name in self.formats:
            return self.formats[name]
        if name == "token_embd.weight":
            return self.embd_format
        if name == "output.weight":
            return self.output_format
        return self.proj_format

    def matrix_shapes(self) -> dict:
        """name -> (rows, cols) for every quantized matrix of the model."""
        H, F, qw, kvw = self.hidden, self.ffn, self.q_width, self.kv_width
        shapes = {"token_embd.weight": (self.vocab, H)}
        if not self.tied_embeddings:
            shapes["output.weight"] = (self.vocab, H)
        for i in range(self.layers):
            p = f"blk.{i}."
            shapes.update({p + "attn_q.weight": (qw, H), p + "attn_k.weight": (kvw, H), p + "attn_v.weight": (kvw, H),
                           p + "attn_output.weight": (H, qw), p + "ffn_gate.weight": (F, H),
                           p + "ffn_up.weight": (F, H), p + "ffn_down.weight": (H, F)})
        return shapes

    def vector_shapes(self) -> dict:
        out = {"output_norm.weight": self.hidden}
        for i in range(self.layers):
            p = f"blk.{i}."
            out[p + "attn_norm.weight"] = self.hidden
            out[p + "ffn_norm.weight"] = self.hidden
            if self.has_bias:
                out[p + "attn_q.bias"] = self.q_width
                out[p + "attn_k.bias"] = self.kv_width
                out[p + "attn_v.bias"] = self.kv_width
        return out

    def weight_bytes(self, include_embedding_table: bool = True) -> int:
        total = 0
        for name, (r, c) in self.matrix_shapes().items():
            if name == "token_embd.weight" and not include_embedding_table:
                continue
            bb = 34 if self.format_of(name) == _lib.Q8_0 else 18
            total += r * (c // 32) * bb
        return total


def qwen2_1_5b() -> ModelSpec:
    """Qwen2-style 1.5B shape, all Q8_0."""
    return ModelSpec(layers=28, hidden=1536, ffn=8960, q_heads=12, kv_heads=2, head_dim=128, vocab=151936,
                     eps=1e-6, rope_base=1e6, name="qwen2-1.5b-shape-q8_0")


def qwen2_7b() -> ModelSpec:
    """Qwen2-style 7B shape, Q4_0 projections, Q8_0 embedding / lm_head."""
    return ModelSpec(layers=28, hidden=3584, ffn=18944, q_heads=28, kv_heads=4, head_dim=128, vocab=152064,
                     eps=1e-6, rope_base=1e6, proj_format=_lib.Q4_0, name="qwen2-7b-shape-q4_0")


def tiny(layers=2, hidden=256, ffn=512, q_heads=4, kv_heads=2, head_dim=64, vocab=1000, proj_format=_lib.Q8_0,
         has_bias=True) -> ModelSpec:
    return ModelSpec(layers=layers, hidden=hidden, ffn=ffn, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim,
                     vocab=vocab, proj_format=proj_format, has_bias=has_bias, name="tiny")


def _tensor_entry(name: str, data, spec: ModelSpec, keep: list):
    """One satori_tensor; `data` is a numpy array (host) or an object with data_ptr() (device)."""
    if hasattr(data, "data_ptr"):
        ptr, nbytes = int(data.data_ptr()), int(data.numel() * data.element_size())
    else:
        arr = np.ascontiguousarray(data)
        keep.append(arr)
        ptr, nbytes = arr.ctypes.data, arr.nbytes
    t = _lib.Tensor()
    bname = name.encode()
    keep.append(bname)
    t.name = bname
    t.data = ptr
    t.bytes = nbytes
    mshapes = spec.matrix_shapes()
    if name in mshapes:
        t.format = spec.format_of(name)
        t.rows, t.cols = mshapes[name]
    else:
        t.format = -1
        t.rows, t.cols = nbytes // 4, 1
    return t


def build_desc(spec: ModelSpec, tensors: dict):
    keep: list = []
    names = list(tensors)
    arr = (_lib.Tensor * len(names))()
    for i, n in enumerate(names):
        arr[i] = _tensor_entry(n, tensors[n], spec, keep)
    d = _lib.ModelDesc()
    d.layers, d.hidden, d.ffn = spec.layers, spec.hidden, spec.ffn
    d.q_heads, d.kv_heads, d.head_dim, d.vocab = spec.q_heads, spec.kv_heads, spec.head_dim, spec.vocab
    d.rms_epsilon, d.rope_base = spec.eps, spec.rope_base
    d.tied_embeddings = int(spec.tied_embeddings)
    d.n_tensors = len(names)
    d.tensors = C.cast(arr, C.POINTER(_lib.Tensor))
    keep.append(arr)
    return d, keep


def nccl_unique_id() -> bytes:
    """The 128-byte NCCL id rank 0 creates and sends to every rank of a sharded session."""
    buf = C.create_string_buffer(128)
    check(_lib.lib().satori_nccl_unique_id(buf), "nccl_unique_id")
    return buf.raw


def broadcast_nccl_id(group=None) -> bytes:
    """Rank 0's NCCL id delivered to every rank of a torch.distributed group (the group only carries
    the 128 bytes; the session's exchanges run on its own NCCL communicator)."""
    import torch.distributed as dist
    obj = [nccl_unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    return obj[0]


def shard_ranges(spec: ModelSpec, rank: int, world: int) -> dict:
    """Rows and heads rank `rank` of `world` computes in a sharded session (mirrors session_plan_shards):
    contiguous row blocks of every projection, query heads [q0, q1) and the KV heads they read."""
    if world == 1:
        return {"hidden": (0, spec.hidden), "ffn": (0, spec.ffn), "vocab": (0, spec.vocab),
                "q_heads": (0, spec.q_heads), "kv_heads": (0, spec.kv_heads)}
    if spec.hidden % world or spec.ffn % world or spec.vocab % world or spec.q_heads < world:
        raise NotSupportedError(_lib.ERR_NOT_SUPPORTED, "shape does not shard over %d ranks" % world)
    group = spec.q_heads // spec.kv_heads
    qa, qb = rank * spec.q_heads // world, (rank + 1) * spec.q_heads // world
    step = lambda n: (rank * (n // world), (rank + 1) * (n // world))
    return {"hidden": step(spec.hidden), "ffn": step(spec.ffn), "vocab": step(spec.vocab), "q_heads": (qa, qb),
            "kv_heads": (qa // group, (qb - 1) // group + 1)}


class CudaDenseSession:
    """IInferenceSession over the GPU (DenseSession.cs).  Not thread-safe, like the reference."""

    def __init__(self, spec: ModelSpec, tensors: dict, context_length: int, ctx: Context | None = None,
                 rank: int = 0, world: int = 1, nccl_id: bytes | None = None):
        if context_length <= 0:
            raise ArgumentError(_lib.ERR_ARGUMENT, "contextLength must be positive")
        self.ctx = ctx or default_context()
        self.spec = spec
        self._h = _vp()
        desc, keep = build_desc(spec, tensors)
        h = _vp()
        if world == 1:
            check(_lib.lib().satori_session_create(self.ctx.handle, C.byref(desc), context_length, C.byref(h)),
                  "session_create")
        else:
            idbuf = C.create_string_buffer(bytes(nccl_id), 128)
            check(_lib.lib().satori_session_create_sharded(self.ctx.handle, C.byref(desc), context_length, rank, world,
                                                           idbuf, C.byref(h)), "session_create_sharded")
        del keep
        self._h = h
        self.context_length = context_length
        self.vocab = spec.vocab

    @classmethod
    def _adopt(cls, handle, ctx: Context, context_length: int, shape: dict):
        """Wraps a session handle created by a native loader (satori_session_create_from_gguf)."""
        s = cls.__new__(cls)
        s.ctx = ctx
        s._h = handle
        s.context_length = context_length
        s.vocab = shape["vocab"]
        s.spec = ModelSpec(layers=shape["layers"], hidden=shape["hidden"], ffn=shape["ffn"],
                           q_heads=shape["q_heads"], kv_heads=shape["kv_heads"], head_dim=shape["head_dim"],
                           vocab=shape["vocab"], eps=shape["rms_epsilon"], rope_base=shape["rope_base"],
                           tied_embeddings=shape["tied_embeddings"], name="gguf")
        return s

    @property
    def handle(self):
        if not self._h:
            raise DisposedError(_lib.ERR_DISPOSED, "Cannot access a disposed object.")
        return self._h

    @property
    def position(self) -> int:
        p = C.c_int()
        check(_lib.lib().satori_session_position(self.handle, C.byref(p)), "position")
        return p.value

    def append(self, token: int, want_logits: bool = True):
        """DenseSession.Append: returns (logits or None, greedy token)."""
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        arg = C.c_int()
        check(_lib.lib().satori_session_append(self.handle, int(token),
                                               logits.ctypes.data if want_logits else None, C.byref(arg)), "append")
        return logits, arg.value

    def forward(self, tokens, logits: np.ndarray | None = None, tensor_cores: bool = False) -> np.ndarray:
        """IInferenceSession.Forward: appends every token, writes the last position's logits.

        tensor_cores=True prefills all but the last token in chunks on the tensor cores
        (satori_session_forward_tensor): not bit-exact, within FP32 rounding of the per-token path."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.size == 0:
            raise ArgumentError(_lib.ERR_ARGUMENT, "At least one token is required.")
        out = np.empty(self.vocab, np.float32)
        arg = C.c_int()
        fn = _lib.lib().satori_session_forward_tensor if tensor_cores else _lib.lib().satori_session_append_tokens
        check(fn(self.handle, t.ctypes.data, t.size, out.ctypes.data, C.byref(arg)), "forward")
        if logits is not None:
            logits[:] = out
            return logits
        return out

    def prefill(self, tokens, tensor_cores: bool = False) -> int:
        """Appends every token without copying logits back; returns the last greedy token."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        arg = C.c_int()
        fn = _lib.lib().satori_session_forward_tensor if tensor_cores else _lib.lib().satori_session_append_tokens
        check(fn(self.handle, t.ctypes.data, t.size, None, C.byref(arg)), "prefill")
        return arg.value

    def generate(self, first: int, count: int) -> np.ndarray:
        """Greedy decode: appends `first`, then feeds back each argmax on the device."""
        out = np.empty(count, np.int32)
        check(_lib.lib().satori_session_generate(self.handle, int(first), int(count), out.ctypes.data), "generate")
        return out

    def stage(self, which: int) -> np.ndarray:
        n = self.vocab if which == 2 else self.spec.hidden
        out = np.empty(n, np.float32)
        check(_lib.lib().satori_session_stage(self.handle, which, out.ctypes.data, n), "stage")
        return out

    def reset(self) -> None:
        check(_lib.lib().satori_session_reset(self.handle), "reset")

    def rewind(self, position: int) -> None:
        """Drops the positions at and after `position`; the earlier cached K/V stay."""
        check(_lib.lib().satori_session_rewind(self.handle, int(position)), "rewind")

    def info(self) -> dict:
        """kernels per decode step, weight bytes held here, K/V bytes per cached position."""
        k, w, kv = C.c_int(), C.c_size_t(), C.c_size_t()
        check(_lib.lib().satori_session_info(self.handle, C.byref(k), C.byref(w), C.byref(kv)), "info")
        return {"kernels_per_step": k.value, "weight_bytes": w.value, "kv_bytes_per_position": kv.value}

    def dispose(self) -> None:
        if self._h:
            _lib.lib().satori_session_destroy(self._h)
            self._h = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass
