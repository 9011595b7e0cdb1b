"""The native GGUF v3 reader (satori_gguf_open, host code: no GPU) against the reference's own GGUF
fixtures and its structure tests (tests/Satori.Numerics.Tests/GgufTests.cs, GgufStructureTests.cs).

InvalidDataException maps to InvalidDataError, NotSupportedException to NotSupportedError."""
import math
import struct

import numpy as np
import pytest

import gguf_util as G
from golden_util import golden


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


def _file(tmp_path, data: bytes, name="t.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


FILES = golden()["gguf_v1_files"]["files"]


@pytest.mark.parametrize("name,type_id,length,offset", [("q4_0", 2, 18, 160), ("q8_0", 8, 34, 160),
                                                        ("f32", 0, 12, 128), ("f16", 1, 6, 128)])
def test_golden_catalogue(sat, oracle_lib, tmp_path, name, type_id, length, offset):
    """GgufTests.GoldenCatalogueAndScopedBounds (GgufTests.cs:31-47) and the fixture manifest."""
    f = FILES[name + ".gguf"]
    with sat.GgufFile(_file(tmp_path, bytes.fromhex(f["hex"]))) as g:
        assert list(g.tensors) == [f["tensor_name"]] == ["weights"]
        t = g.tensors["weights"]
        assert (t.type, t.byte_length, t.offset) == (type_id, length, offset)
        assert list(t.dimensions) == f["dimensions"]
        assert len(g.metadata) == f["metadata_count"]
        assert g.read_scalar("general.architecture") == "llama"
        payload = g.read_tensor("weights")
        assert payload.size == f["payload_bytes"]
        if type_id in (2, 8):
            assert g.read_scalar("general.quantization_version") == 2
            decoded = oracle_lib.q_decode_row(payload, t.dimensions[0], 0 if type_id == 8 else 1)
        else:
            decoded = payload.view(np.float32 if type_id == 0 else np.float16).astype(np.float32)
        assert decoded.tolist() == f["decoded_weights"]
        # scoped bounds: a window past the payload is refused, an empty one at its end is empty
        with pytest.raises(sat.ArgumentError):
            g.read_tensor("weights", length, 1)
        assert g.read_tensor("weights", length, 0).size == 0
        assert g.read_tensor("weights", 1, 2).tolist() == payload[1:3].tolist()
    with pytest.raises(sat.DisposedError):
        g.read_tensor("weights", 0, 1)


def test_every_truncation_rejects(sat, tmp_path):
    """GgufTests.EveryTruncationRejectsWithoutPublishingCatalogue (GgufTests.cs:49-58)."""
    raw = bytes.fromhex(FILES["q8_0.gguf"]["hex"])
    for n in range(len(raw)):
        with pytest.raises(sat.InvalidDataError):
            sat.GgufFile(_file(tmp_path, raw[:n], f"t{n}.gguf"))


def test_mutations_and_unsupported_version(sat, tmp_path):
    """GgufTests.MutatedStructureAndUnsupportedVersionReject (GgufTests.cs:60-74)."""
    raw = bytes.fromhex(FILES["q8_0.gguf"]["hex"])
    for index in (0, 32, 45, 137):
        b = bytearray(raw)
        b[index] = 0xFF
        with pytest.raises(sat.InvalidDataError):
            sat.GgufFile(_file(tmp_path, bytes(b), f"m{index}.gguf"))
    b = bytearray(raw)
    b[4:8] = struct.pack("<I", 2)
    with pytest.raises(sat.NotSupportedError):
        sat.GgufFile(_file(tmp_path, bytes(b), "v2.gguf"))


def test_repeated_reads_are_stable(sat, tmp_path):
    """GgufTests.RepeatedMappedStringReadsKeepNamesAndScalarTypesStable (GgufTests.cs:8-19)."""
    path = _file(tmp_path, bytes.fromhex(FILES["q8_0.gguf"]["hex"]))
    for _ in range(200):
        with sat.GgufFile(path) as g:
            assert g.read_scalar("general.architecture") == "llama"
            assert g.read_scalar("general.quantization_version") == 2
            assert g.tensors["weights"].type == 8


def _sparse(tmp_path, name, length, head=b"", tail_at=None, tail=b""):
    """A file of `length` bytes written only where given (MappedFileFixture with a sparse body)."""
    p = tmp_path / name
    with open(p, "wb") as f:
        f.write(head)
        if tail_at is not None:
            f.seek(tail_at)
            f.write(tail)
        f.truncate(length)
    return str(p)


def test_oversized_sparse_file_rejects_before_mapping(sat, tmp_path):
    """GgufStructureTests.OversizedSparseFileRejectsBeforeMapping (GgufStructureTests.cs:57-63)."""
    try:
        path = _sparse(tmp_path, "huge.gguf", (1 << 40) + 1)
    except OSError as e:   # a file system without sparse files of that size
        pytest.skip(f"cannot create a sparse 1 TiB file here: {e}")
    with pytest.raises(sat.NotSupportedError, match="File limit"):
        sat.GgufFile(path)


def test_sparse_tensor_beyond_two_gib(sat, tmp_path):
    """GgufStructureTests.SparseTensorBeyondTwoGiBUsesInt64Windows (GgufStructureTests.cs:84-99): offsets
    past 2^31 are 64-bit, and a window reaching past a tensor is refused."""
    first = 1 << 31
    head = G.prefix(32, tensors=[("large", [first // 4], G.T_F32, 0), ("tail", [1], G.T_F32, first)])
    try:
        path = _sparse(tmp_path, "big.gguf", len(head) + first + 32, head, len(head) + first, bytes([1, 2, 3, 4]))
    except OSError as e:
        pytest.skip(f"cannot create a sparse 2 GiB file here: {e}")
    with sat.GgufFile(path) as g:
        assert g.tensors["tail"].offset == len(head) + first
        assert g.read_tensor("tail", 0, 4).tolist() == [1, 2, 3, 4]
        with pytest.raises(sat.ArgumentError):
            g.read_tensor("large", first - 1, 2)


def test_closed_file_refuses_access(sat, tmp_path):
    g = sat.GgufFile(_file(tmp_path, bytes.fromhex(FILES["q8_0.gguf"]["hex"])))
    g.close()
    with pytest.raises(sat.DisposedError):
        g.read_scalar("general.architecture")


def _scalar_value(t):
    return {0: 17, 1: -17, 2: 17, 3: -17, 4: 17, 5: -17, 6: float("inf"), 7: 1, 8: "è\0漢", 9: (G.BOOL, [0, 1]),
            10: 17, 11: -17, 12: float("nan")}[t]


@pytest.mark.parametrize("alignment", [8, 64, 4096])
def test_mixed_scalar_types_and_flat_arrays(sat, tmp_path, alignment):
    """GgufStructureTests.MixedTensorsAllScalarTypesAndFlatArrays (GgufStructureTests.cs:7-35)."""
    meta = b"".join(G.entry(f"custom.value_{t}", t, _scalar_value(t)) for t in range(13))
    meta += G.entry("custom.empty", G.ARR, (G.STR, []))
    meta += G.entry("custom.strings", G.ARR, (G.STR, ["è\0漢", ""]))
    pre = G.prefix(alignment, meta, 15)
    with sat.GgufFile(_file(tmp_path, G.file_with(pre, len(pre) + alignment * 2 + 3))) as g:
        assert len(g.tensors) == 2 and len(g.metadata) == 17
        assert g.read_scalar("custom.value_8") == "è\0漢"
        assert g.read_scalar("custom.value_4") == 17
        assert g.read_scalar("custom.value_11") == -17
        assert g.read_scalar("custom.value_6") == math.inf
        assert math.isnan(g.read_scalar("custom.value_12"))
        assert g.read_scalar("custom.value_7") is True
        assert g.metadata["custom.empty"].element_count == 0
        assert g.metadata["custom.strings"].element_count == 2
        assert g.tensors["second"].offset == len(pre) + alignment
        with pytest.raises(sat.ArgumentError):
            g.read_scalar("custom.strings")


@pytest.mark.parametrize("split_count,split_no,rejected", [(0, 0, False), (1, 0, False), (2, 0, True), (1, 1, True)])
def test_split_count(sat, tmp_path, split_count, split_no, rejected):
    """GgufStructureTests.SplitCountZeroIsTreatedAsUnsharded (GgufStructureTests.cs:65-82)."""
    meta = G.entry("split.count", G.U16, split_count) + G.entry("split.no", G.U16, split_no)
    pre = G.prefix(32, meta, 2)
    path = _file(tmp_path, G.file_with(pre, len(pre) + 64))
    if rejected:
        with pytest.raises(sat.NotSupportedError):
            sat.GgufFile(path)
    else:
        with sat.GgufFile(path) as g:
            assert len(g.tensors) == 2


@pytest.mark.parametrize("defect", ["bool", "key", "duplicate", "utf8", "typed"])
def test_invalid_metadata_rejects(sat, tmp_path, defect):
    """GgufStructureTests.InvalidMetadataRejects (GgufStructureTests.cs:100-118)."""
    key = {"key": "BAD.key", "duplicate": "general.architecture", "typed": "general.file_type"}.get(defect, "custom.test")
    meta = G.gstr(key)
    if defect == "utf8":
        meta += struct.pack("<IQ", 8, 1) + b"\xff"
    else:
        meta += struct.pack("<I", 7) + bytes([2 if defect == "bool" else 1])
    pre = G.prefix(32, meta, 1)
    with pytest.raises(sat.InvalidDataError):
        sat.GgufFile(_file(tmp_path, G.file_with(pre, len(pre) + 64)))


@pytest.mark.parametrize("defect", ["overlap", "overflow", "zero", "unaligned", "duplicate"])
def test_invalid_tensor_structure_rejects(sat, tmp_path, defect):
    """GgufStructureTests.InvalidTensorStructureRejects (GgufStructureTests.cs:120-139)."""
    tensors = {"overlap": [("a", [32], 0, 0), ("b", [1], 0, 32)],
               "overflow": [("a", [2 ** 63 - 1, 2], 0, 0)],
               "zero": [("a", [0], 0, 0)],
               "unaligned": [("a", [1], 0, 1)],
               "duplicate": [("a", [1], 0, 0), ("a", [1], 0, 32)]}[defect]
    pre = G.prefix(32, tensors=tensors)
    with pytest.raises(sat.InvalidDataError):
        sat.GgufFile(_file(tmp_path, G.file_with(pre, len(pre) + 256)))


def test_gap_and_reverse_order_are_unsupported(sat, tmp_path):
    """GgufStructureTests.GapAndReversePhysicalOrderAreUnsupportedRatherThanCorrupt (:141-152)."""
    for offsets in ((32, 64), (32, 0)):
        pre = G.prefix(32, tensors=[("a", [1], 0, offsets[0]), ("b", [1], 0, offsets[1])])
        with pytest.raises(sat.NotSupportedError):
            sat.GgufFile(_file(tmp_path, G.file_with(pre, len(pre) + 128)))


def test_k_quant_types_are_accepted(sat, tmp_path):
    """GgufStructureTests.KQuantizedTypesAreAcceptedByTheExtendedProfile (:154-170)."""
    meta = G.entry("general.quantization_version", G.U32, 2)
    pre = G.prefix(32, meta, 1, [("q4k", [256, 2], 12, 0), ("q6k", [256, 1], 14, 288)])
    with sat.GgufFile(_file(tmp_path, G.file_with(pre, len(pre) + 512))) as g:
        assert (g.tensors["q4k"].type, g.tensors["q6k"].type) == (12, 14)
        assert (g.tensors["q4k"].byte_length, g.tensors["q6k"].byte_length) == (288, 210)


def test_missing_quantization_version_and_unsupported_type(sat, tmp_path):
    pre = G.prefix(32, tensors=[("q", [32], 8, 0)])
    with pytest.raises(sat.InvalidDataError):
        sat.GgufFile(_file(tmp_path, G.file_with(pre, len(pre) + 64)))
    pre = G.prefix(32, G.entry("general.quantization_version", G.U32, 2), 1, [("q", [32], 3, 0)])
    with pytest.raises(sat.NotSupportedError):
        sat.GgufFile(_file(tmp_path, G.file_with(pre, len(pre) + 64)))


def test_model_description_from_metadata(sat, tmp_path):
    """DenseTransformerAdapter.Validate over a qwen2 container: shape from {arch}.* keys, vocabulary from
    token_embd.weight, untied output, optional biases; a missing tensor is a capability gap."""
    from model_util import synthetic_tensors
    spec = sat.tiny()
    tensors = synthetic_tensors(spec, 3)
    data = G.model_gguf(spec, tensors)
    with sat.GgufFile(_file(tmp_path, data)) as g:
        d = g.model_desc()
        assert (d["layers"], d["hidden"], d["ffn"], d["q_heads"], d["kv_heads"], d["head_dim"], d["vocab"]) == \
            (spec.layers, spec.hidden, spec.ffn, spec.q_heads, spec.kv_heads, spec.head_dim, spec.vocab)
        assert d["rope_base"] == spec.rope_base and not d["tied_embeddings"]
        assert d["tensors"] == len(tensors)
        assert np.array_equal(g.read_tensor("blk.1.ffn_down.weight"), tensors["blk.1.ffn_down.weight"])
    broken = dict(tensors)
    del broken["blk.0.attn_k.weight"]
    with sat.GgufFile(_file(tmp_path, G.model_gguf(spec, broken), "broken.gguf")) as g:
        with pytest.raises(sat.NotSupportedError):
            g.model_desc()


def _qwen_container(tmp_path, name, arch="qwen2", embedding=64, heads=2, heads_kv=1, ffn=64, vocab=10, layers=2,
                    key_length=None, drop_meta=(), shapes=None):
    """A qwen-style container with Q8_0 matrices (zero payload) and F32 norms in canonical order, for the
    model-description rules (ModelDescriptorTests' Qwen2 helper, written as a GGUF file)."""
    head_dim = key_length or max(1, embedding // heads)
    q, kv = heads * head_dim, heads_kv * head_dim
    meta = [(f"{arch}.block_count", G.U32, layers), (f"{arch}.embedding_length", G.U32, embedding),
            (f"{arch}.feed_forward_length", G.U32, ffn), (f"{arch}.attention.head_count", G.U32, heads),
            (f"{arch}.attention.head_count_kv", G.U32, heads_kv),
            (f"{arch}.attention.layer_norm_rms_epsilon", G.F32, 1e-6), (f"{arch}.rope.freq_base", G.F32, 1e6),
            ("general.quantization_version", G.U32, 2)]
    if key_length is not None:
        meta.append((f"{arch}.attention.key_length", G.U32, key_length))
    meta = [m for m in meta if m[0].split(".", 1)[1] not in drop_meta]
    want = [("token_embd.weight", [embedding, vocab]), ("output_norm.weight", [embedding])]
    for l in range(layers):
        p = f"blk.{l}."
        want += [(p + "attn_norm.weight", [embedding]), (p + "attn_q.weight", [embedding, q]),
                 (p + "attn_k.weight", [embedding, kv]), (p + "attn_v.weight", [embedding, kv]),
                 (p + "attn_output.weight", [q, embedding]), (p + "ffn_norm.weight", [embedding]),
                 (p + "ffn_gate.weight", [embedding, ffn]), (p + "ffn_up.weight", [embedding, ffn]),
                 (p + "ffn_down.weight", [ffn, embedding])]
    want = [(n, (shapes or {}).get(n, d)) for n, d in want]
    tensors, off = [], 0
    for n, dims in want:
        t = G.T_Q8_0 if len(dims) == 2 else G.T_F32
        nbytes = dims[0] // 32 * 34 * dims[1] if t == G.T_Q8_0 else 4 * dims[0]
        tensors.append((n, dims, t, off))
        off = (off + nbytes + 31) // 32 * 32
    head = G.prefix(32, b"".join(G.entry(*m) for m in meta), len(meta), tensors, arch=arch)
    return _file(tmp_path, G.file_with(head, len(head) + off), name)


def test_dense_adapter_derives_shape(sat, tmp_path):
    """ModelDescriptorTests.DenseAdapterDerivesShapeAndReportsNoGaps (ModelDescriptorTests.cs:11-23): the head
    length is embedding / heads when no key_length is declared; the vocabulary comes from token_embd."""
    with sat.GgufFile(_qwen_container(tmp_path, "a.gguf")) as g:
        d = g.model_desc()
    assert (d["layers"], d["hidden"], d["head_dim"], d["kv_heads"], d["vocab"]) == (2, 64, 32, 1, 10)
    assert d["tied_embeddings"]          # no output.weight: the embedding is the output projection
    assert d["tensors"] == 2 + 2 * 9


def test_explicit_key_length_overrides_hidden_over_heads(sat, tmp_path):
    """ModelDescriptorTests.ExplicitKeyLengthOverridesHiddenOverHeads (ModelDescriptorTests.cs:25-35)."""
    with sat.GgufFile(_qwen_container(tmp_path, "k.gguf", layers=1, key_length=48)) as g:
        assert g.model_desc()["head_dim"] == 48


def test_incompatible_shape_is_reported(sat, tmp_path):
    """ModelDescriptorTests.IncompatibleShapeIsReported (ModelDescriptorTests.cs:37-48): the wrong tensor is named."""
    path = _qwen_container(tmp_path, "s.gguf", layers=1, shapes={"blk.0.attn_q.weight": [64, 999]})
    with sat.GgufFile(path) as g:
        with pytest.raises(sat.NotSupportedError, match="blk.0.attn_q.weight"):
            g.model_desc()


def test_indivisible_embedding_without_key_length_is_reported(sat, tmp_path):
    """ModelDescriptorTests.UndeclaredHeadLengthWithIndivisibleEmbeddingIsReported (ModelDescriptorTests.cs:50-56)."""
    path = _qwen_container(tmp_path, "i.gguf", embedding=96, heads=5, layers=1,
                           shapes={"blk.0.attn_output.weight": [96, 96]})   # any whole-block width parses
    with sat.GgufFile(path) as g:
        with pytest.raises(sat.NotSupportedError, match="attention.key_length"):
            g.model_desc()


def test_missing_required_metadata_is_reported(sat, tmp_path):
    """ModelDescriptorTests.MissingRequiredMetadataIsReported (ModelDescriptorTests.cs:58-70)."""
    drop = ("embedding_length", "feed_forward_length", "attention.head_count", "attention.head_count_kv")
    with sat.GgufFile(_qwen_container(tmp_path, "m.gguf", layers=1, drop_meta=drop)) as g:
        with pytest.raises(sat.NotSupportedError, match="embedding_length"):
            g.model_desc()


@pytest.mark.parametrize("arch,supported", [("qwen3", True), ("mysterymoe", False)])
def test_architecture_adapter(sat, tmp_path, arch, supported):
    """ModelDescriptorTests.UnknownArchitectureHasNoAdapter (ModelDescriptorTests.cs:72-77): qwen2 and qwen3
    resolve, any other architecture has no dense adapter."""
    with sat.GgufFile(_qwen_container(tmp_path, arch + ".gguf", arch=arch, layers=1)) as g:
        if supported:
            assert g.model_desc()["layers"] == 1
        else:
            with pytest.raises(sat.NotSupportedError):
                g.model_desc()
