"""The model shapes the session tests and the bench build on, pinned to the reference's records of two real
models (no GPU):

* the GGUF catalogue of qwen2.5-coder-1.5b-q8_0 and the plan the reference's benchmark reported for it
  at context 2048 (docs/scouting/inventories/qwen2.5-coder-1.5b-q8_0.json,
  docs/benchmarks/qwen-2026-10-13/qwen2.5-coder-1.5b-q8_0-ctx2048.json:14-31) against ``qwen2_1_5b()``,
  tensor by tensor;
* the catalogue of qwen2.5-coder-7b-q4_0 against ``qwen2_7b()``: every layer tensor is identical; the
  embedding and the output projection have the same dimensions, in Q8_0 as the benchmark configuration
  states rather than the file's Q4_0 / Q6_K;
* the native loader (``satori_gguf_open`` + ``satori_gguf_model_desc``) on a sparse container holding each
  real catalogue (those two, the 7B Q4_K_M file and the qwen3 4B Q8_0 file): it derives each model's
  description from the recorded metadata and tensors.
"""
import struct

import pytest

import gguf_util as G
from golden_util import golden

INV = golden()["model_inventories"]
_GGUF_TYPE = {0: 8, 1: 2}          # this library's Q8_0 / Q4_0 -> GGUF type ids


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


def _spec_catalogue(spec):
    """name -> (GGUF type id, GGUF dimensions, byte length) of a spec's tensors."""
    out = {}
    for name, (rows, cols) in spec.matrix_shapes().items():
        fmt = spec.format_of(name)
        out[name] = (_GGUF_TYPE[fmt], [cols, rows], rows * (cols // 32) * (34 if fmt == 0 else 18))
    for name, n in spec.vector_shapes().items():
        out[name] = (0, [n], 4 * n)
    return out


def test_1_5b_spec_is_the_real_models_catalogue(sat):
    inv = INV["qwen2.5-coder-1.5b-q8_0"]
    ours = _spec_catalogue(sat.qwen2_1_5b())
    theirs = {name: (t, dims, length) for name, t, dims, _, length in inv["tensors"]}
    assert len(ours) == inv["tensor_count"] == 339
    assert ours == theirs
    assert sum(v[2] for v in ours.values()) == inv["total_tensor_bytes"] == inv["plan_ctx2048"]["weight_bytes"]


def test_1_5b_spec_matches_the_reference_plan(sat):
    plan = INV["qwen2.5-coder-1.5b-q8_0"]["plan_ctx2048"]
    spec, shape = sat.qwen2_1_5b(), plan["shape"]
    assert (spec.layers, spec.hidden, spec.ffn, spec.q_heads, spec.kv_heads, spec.head_dim, spec.vocab) == \
        (shape["Layers"], shape["EmbeddingLength"], shape["FeedForwardLength"], shape["HeadCount"],
         shape["HeadCountKv"], shape["HeadDim"], shape["VocabularySize"])
    assert spec.tied_embeddings == shape["TiedEmbeddings"]
    # ModelPlanner's KV state: layers x {K, V} x context x kv_width x 4 bytes, the session's cache.
    assert spec.layers * 2 * plan["context"] * spec.kv_width * 4 == plan["state_bytes"]


def test_7b_spec_layers_are_the_real_models(sat):
    inv = INV["qwen2.5-coder-7b-q4_0"]
    ours = _spec_catalogue(sat.qwen2_7b())
    theirs = {name: (t, dims, length) for name, t, dims, _, length in inv["tensors"]}
    assert set(ours) == set(theirs) and len(ours) == inv["tensor_count"]
    for name in ours:
        if name in ("token_embd.weight", "output.weight"):
            assert ours[name][0] == 8 and ours[name][1] == theirs[name][1] == [3584, 152064]
        else:
            assert ours[name] == theirs[name], name


def _catalogue_container(tmp_path, inv, name):
    """A sparse GGUF file with the model's recorded metadata and tensor catalogue; payload bytes absent."""
    types = {"UInt8": G.U8, "Int8": G.I8, "UInt16": G.U16, "Int16": G.I16, "UInt32": G.U32, "Int32": G.I32,
             "Float32": G.F32, "Bool": G.BOOL, "String": G.STR, "UInt64": G.U64, "Int64": G.I64, "Float64": G.F64}
    entries = []
    for key, type_name, value in inv["metadata"]:
        if key in ("general.architecture", "general.alignment"):
            continue
        t = types[type_name]
        entries.append(G.entry(key, t, int(value) if t == G.BOOL else value))
    tensors = [(n, dims, t, off) for n, t, dims, off, _ in inv["tensors"]]
    arch = next(value for key, _, value in inv["metadata"] if key == "general.architecture")
    head = G.prefix(inv["alignment"], b"".join(entries), len(entries), tensors, arch=arch)
    end = max(off + length for _, _, _, off, length in inv["tensors"])
    end = (end + inv["alignment"] - 1) // inv["alignment"] * inv["alignment"]
    path = tmp_path / name
    try:
        with open(path, "wb") as fh:
            fh.write(head)
            fh.truncate(len(head) + end)
    except OSError as e:
        pytest.skip(f"cannot create a sparse model-sized file here: {e}")
    return str(path)


def _expected_description(inv):
    """The description DenseTransformerAdapter derives, read off the recorded catalogue: the {arch}.* keys,
    head length = key_length when declared (else embedding / heads), vocabulary = token_embd's rows, tied
    when there is no output.weight."""
    meta = {key: value for key, _, value in inv["metadata"]}
    arch = meta["general.architecture"]
    dims = {name: d for name, _, d, _, _ in inv["tensors"]}
    hidden, heads = meta[f"{arch}.embedding_length"], meta[f"{arch}.attention.head_count"]
    head_dim = meta.get(f"{arch}.attention.key_length", hidden // heads)
    return ((meta[f"{arch}.block_count"], hidden, meta[f"{arch}.feed_forward_length"], heads,
             meta[f"{arch}.attention.head_count_kv"], head_dim, dims["token_embd.weight"][1]),
            "output.weight" not in dims, arch)


@pytest.mark.parametrize("model,expected", [
    ("qwen2.5-coder-1.5b-q8_0", (28, 1536, 8960, 12, 2, 128, 151936)),
    ("qwen2.5-coder-7b-q4_0", (28, 3584, 18944, 28, 4, 128, 152064)),
    ("qwen2.5-coder-7b-q4_k_m", (28, 3584, 18944, 28, 4, 128, 152064)),
    ("qwen3-4b-q8_0", None),
])
def test_native_loader_derives_the_real_models_shape(sat, tmp_path, model, expected):
    """Q8_0, Q4_0 with a Q6_K output, the K-quant mix of Q4_K_M, and qwen3 (per-head q/k norms, a declared
    key length, tied embeddings): every tensor of each catalogue enters the description."""
    inv = INV[model]
    want, tied, arch = _expected_description(inv)
    if expected is not None:
        assert want == expected
    with sat.GgufFile(_catalogue_container(tmp_path, inv, model + ".gguf")) as g:
        assert len(g.tensors) == inv["tensor_count"]
        d = g.model_desc()
        assert g.read_scalar(f"{arch}.rope.freq_base") == pytest.approx(1e6)
    assert (d["layers"], d["hidden"], d["ffn"], d["q_heads"], d["kv_heads"], d["head_dim"], d["vocab"]) == want
    assert d["tied_embeddings"] == tied
    assert d["tensors"] == inv["tensor_count"]
    assert d["rope_base"] == 1e6
    assert struct.pack("<f", d["rms_epsilon"]) == struct.pack("<f", 1e-6)
