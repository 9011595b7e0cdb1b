"""Regenerate ``tests/golden/reference_fixtures.json`` from the reference project's own fixtures.

Run in a container that has the reference checked out::

    python tests/golden/make_golden.py /path/to/reference

The reference tree does not travel to the GPU box, so the vectors its tests pin are copied
here once, as data, together with where each came from:

* ``fixtures/gguf/v1/{q8_0,q4_0}.gguf`` + ``manifest.json`` -- the payload bytes of the one
  32-weight tensor (at ``data_start``), its decoded weights and the ones-vector dot (-8),
  pinned by QuantizedTests.cs:9-25 and QuantizedAvx2Tests.cs:52-65.
* ``fixtures/operators/transformer-v1.json`` -- RmsNorm (eps 1e-5), interleaved Rope
  (head 48, position 37), SwiGlu and 2x48 MHA over 7 tokens, pinned by TransformerOpsTests.cs:8-25.
* ``fixtures/operators/transformer-v2.json`` -- GQA 4q/2kv x 8 over 3 tokens, half-split RoPE
  (base 1e6 and a partial rotary case), per-head RmsNorm and bias add, pinned by
  QwenOperatorTests.cs:28-94.
* ``fixtures/operators/attention-boundaries-v1.json`` -- 6 heads x 48 over 1, 2, 32, 64 and 128
  tokens.  Only the expected outputs are stored; the inputs are the deterministic formulas of
  tools/attention_reference.py:4-6, restated in tests/golden_util.py.
* The Ternary2 encoding KAT (Ternary2Tests.cs:9-22) and the STQ2 header KAT
  (MappedTernary2Tests.cs:40-46) are byte strings stated in those tests; they are copied too.
* ``docs/scouting/inventories/{qwen2.5-coder-1.5b-q8_0,qwen2.5-coder-7b-q4_0,qwen2.5-coder-7b-q4_k_m,
  qwen3-4b-q8_0}.json`` -- the GGUF catalogues of four real models (scalar metadata, every tensor's name /
  type / dimensions / offset / length) and the plan
  of ``docs/benchmarks/qwen-2026-10-13/qwen2.5-coder-1.5b-q8_0-ctx2048.json`` (shape, weight and KV
  state bytes), for the model-shape and native-loader tests.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_fixtures.json")


def main(ref: str, out_path: str = OUT) -> None:
    gguf_dir = os.path.join(ref, "fixtures", "gguf", "v1")
    manifest = json.load(open(os.path.join(gguf_dir, "manifest.json")))
    gguf = {}
    for entry in manifest["fixtures"]:
        if entry["tensor_type_id"] not in (2, 8):
            continue
        raw = open(os.path.join(gguf_dir, entry["file"]), "rb").read()
        start = entry["data_start"] + entry["relative_offset"]
        payload = raw[start:start + entry["payload_bytes"]]
        cols, rows = entry["dimensions"]  # GGUF lists the fastest dimension first
        gguf["q8_0" if entry["tensor_type_id"] == 8 else "q4_0"] = {
            "source": f"fixtures/gguf/v1/{entry['file']} (sha256 {entry['sha256']})",
            "rows": rows, "cols": cols, "payload_hex": payload.hex(),
            "decoded_weights": entry["decoded_weights"], "ones_dot_product": entry["ones_dot_product"],
        }

    # The whole fixture files (160-224 bytes each), for the native GGUF reader's tests.
    gguf_files = {}
    for entry in manifest["fixtures"]:
        raw = open(os.path.join(gguf_dir, entry["file"]), "rb").read()
        gguf_files[entry["file"]] = {
            "hex": raw.hex(), "sha256": entry["sha256"], "tensor_name": entry["tensor_name"],
            "tensor_type_id": entry["tensor_type_id"], "dimensions": entry["dimensions"],
            "data_start": entry["data_start"], "payload_bytes": entry["payload_bytes"],
            "alignment": entry["alignment"], "metadata_count": entry["metadata_count"],
            "decoded_weights": entry["decoded_weights"],
        }

    ops = os.path.join(ref, "fixtures", "operators")
    # K-quant fixtures, whole: Q4_K / Q6_K decode and dot (independent FP64), the Q8_K quantizer's exact
    # bytes with the Q4_K x Q8_K product, the Q6_K x Q8_K product, and blocks of two real tensors.
    kquants = {}
    for name in ("q4k-v1", "q6k-v1", "q8k-v1", "q6k-q8k-v1", "k-real-v1"):
        kquants[name.replace("-", "_")] = json.load(open(os.path.join(ops, name + ".json")))
    v1 = json.load(open(os.path.join(ops, "transformer-v1.json")))
    v2 = json.load(open(os.path.join(ops, "transformer-v2.json")))
    ab = json.load(open(os.path.join(ops, "attention-boundaries-v1.json")))
    v1.pop("numpy", None)
    v2.pop("numpy", None)
    v1["params"] = {"rms_epsilon": 1e-5, "rope_head_dim": 48, "rope_position": 37,
                    "attention_head_dim": 48, "attention_tokens": 7,
                    "stated_in": "tests/Satori.Numerics.Tests/TransformerOpsTests.cs:19-24"}

    # Catalogues of two real models as the reference's GGUF inventory recorded them (scalar metadata and
    # every tensor's name, type, dimensions, relative offset and length; the arrays' values are not
    # recorded there), and the plan the reference's benchmark reported for the 1.5B model at context 2048.
    inventories = {}
    for name in ("qwen2.5-coder-1.5b-q8_0", "qwen2.5-coder-7b-q4_0", "qwen2.5-coder-7b-q4_k_m", "qwen3-4b-q8_0"):
        inv = json.load(open(os.path.join(ref, "docs", "scouting", "inventories", name + ".json")))
        meta = [[m["Key"], m["TypeName"], m["Value"]] for m in inv["Metadata"]
                if m["TypeName"] != "Array" and not m["Key"].startswith("tokenizer.chat")]
        inventories[name] = {
            "source": f"docs/scouting/inventories/{name}.json",
            "tensor_count": inv["TensorCount"], "alignment": inv["Alignment"],
            "total_tensor_bytes": inv["TotalTensorBytes"], "metadata": meta,
            "tensors": [[t["Name"], t["TypeId"], t["Dimensions"], t["Offset"], t["ByteLength"]] for t in inv["Tensors"]],
        }
    bench = json.load(open(os.path.join(ref, "docs", "benchmarks", "qwen-2026-10-13",
                                        "qwen2.5-coder-1.5b-q8_0-ctx2048.json")))
    inventories["qwen2.5-coder-1.5b-q8_0"]["plan_ctx2048"] = {
        "source": "docs/benchmarks/qwen-2026-10-13/qwen2.5-coder-1.5b-q8_0-ctx2048.json",
        "context": bench["Context"], "shape": bench["Shape"], "weight_bytes": bench["Plan"]["WeightBytes"],
        "state_bytes": bench["Plan"]["StateBytes"]}

    out = {
        "generated_from": "Satori reference fixtures; regenerate with tests/golden/make_golden.py",
        "model_inventories": inventories,
        "tolerance_operator": {"abs": 2e-6, "rel": 2e-6, "stated_in": "QwenOperatorTests.cs:24; TransformerOpsTests.cs:16"},
        "gguf_v1": gguf,
        "gguf_v1_files": {"source": "fixtures/gguf/v1/*.gguf and manifest.json", "files": gguf_files},
        "kquants": {"source": "fixtures/operators/{q4k,q6k,q8k,q6k-q8k,k-real}-v1.json", **kquants},
        "transformer_v1": v1,
        "transformer_v2": v2,
        "attention_boundaries_v1": {"source": "fixtures/operators/attention-boundaries-v1.json",
                                    "width": 288, "head_dim": 48, "cases": ab["cases"]},
        "ternary2_encoding_kat": {
            "source": "tests/Satori.Numerics.Tests/Ternary2Tests.cs:9-22",
            "weights_nonzero": {"0": 2.0, "1": -2.0}, "rows": 1, "cols": 64, "block_size": 64,
            "expected_hex": "00008" + "03d09" + "00" * 15,
        },
        "stq2_header_kat": {
            "source": "tests/Satori.Numerics.Tests/MappedTernary2Tests.cs:40-46",
            "matrix": {"weights": [1.0], "rows": 1, "cols": 1, "block_size": 64},
            "expected_hex": "53545132" "01002000" "01000000" "01000000"
                            "40000000" "00000000" "14000000" "00000000",
        },
    }
    with open(out_path, "w") as fh:
        json.dump(out, fh, separators=(",", ":"))
        fh.write("\n")
    print(out_path, os.path.getsize(out_path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        sys.exit("usage: python tests/golden/make_golden.py <path to the Satori reference checkout> [output]")
    main(*sys.argv[1:])
