"""Pins the CPU oracle to the reference's own golden vectors and known-answer tests.

The oracle is the checker for every GPU parity test, so it is trusted only after these pass.
Each test names the reference test it restates.
"""
import numpy as np
import pytest

from golden_util import (FLT_MAX, attention_boundary_inputs, bits_equal, critical_cases, gamma_bound, golden,
                         numerical_random, operator_close, q8_critical_cases, q_reference_fp64, t2_bound_ok)


# ----------------------------------------------------------------- GGUF golden files
@pytest.mark.parametrize("fmt_name,fmt", [("q8_0", 0), ("q4_0", 1)])
def test_gguf_golden_decode_and_ones_dot(oracle_lib, fmt_name, fmt):
    """QuantizedTests.GoldenImportedAndOwnedAgreeWithManualDot (QuantizedTests.cs:9-25) and
    QuantizedAvx2Tests.MappedGoldenAutoIsExactAndAllocationFree (:52-65)."""
    g = golden()["gguf_v1"][fmt_name]
    payload = np.frombuffer(bytes.fromhex(g["payload_hex"]), dtype=np.uint8)
    assert oracle_lib.q_validate(payload, 1, 32, fmt) == 0
    np.testing.assert_array_equal(oracle_lib.q_decode_row(payload, 32, fmt), np.array(g["decoded_weights"], np.float32))
    ones = np.ones(32, np.float32)
    for order in ("scalar", "avx2", "avx2_emulated", "batch", "batch_emulated"):
        y = oracle_lib.q_matvec(payload, 1, 32, fmt, ones, order=order)
        assert y[0] == np.float32(g["ones_dot_product"]) == np.float32(-8.0), order


@pytest.mark.parametrize("bits", [0x7C00, 0xFC00, 0x7E00])
@pytest.mark.parametrize("fmt", [0, 1])
def test_nonfinite_scales_rejected(oracle_lib, bits, fmt):
    """QuantizedTests.NonfiniteScalesRejectBeforeCompute (:57-71); Q4Tests.NonfiniteQ4ScaleRejects (:39-47)."""
    payload = np.zeros(34 if fmt == 0 else 18, np.uint8)
    payload[0], payload[1] = bits & 0xFF, bits >> 8
    assert oracle_lib.q_validate(payload, 1, 32, fmt) == oracle_lib.ERR_INVALID_DATA


def test_q_geometry_rejects_partial_blocks(oracle_lib):
    with pytest.raises(oracle_lib.OracleError):
        oracle_lib.q_geometry(1, 33, 0)
    assert oracle_lib.q_geometry(11008, 4096, 1) == (18, 25362432)
    assert oracle_lib.q_geometry(4096, 4096, 0) == (34, 17825792)


# ----------------------------------------------------------------- Q8_0 / Q4_0 arithmetic
def test_q8_critical_cases_within_fp64_bound(oracle_lib):
    """Q8Validation.CriticalCases + Compare (Q8Validation.cs:9-53): every order passes the FP64 bound."""
    for name, rows, cols, payload, x in q8_critical_cases():
        exact, mag = q_reference_fp64(payload, rows, cols, 0, x)
        bound = gamma_bound(cols, mag)
        for order in ("scalar", "avx2", "batch"):
            y = oracle_lib.q_matvec(payload, rows, cols, 0, x, order=order)
            assert np.all(np.abs(y.astype(np.float64) - exact) <= bound), (name, order)


def test_q8_full_signed_range_matches_fp64(oracle_lib):
    """QuantizedTests.Q8FullSignedRangeNegativeSubnormalAndZeroScalesMatchFp64 (:27-55)."""
    rows, cols = 7, 96
    scales = [0.5, -2.0, 0.0, -0.0, 5.960464477539063e-08, 65504.0, 1.0]
    x = np.array([(i % 13 - 6) / 16.0 for i in range(96)], np.float32)
    payload = np.zeros(rows * 3 * 34, np.uint8)
    ref = np.zeros(rows)
    for r in range(rows):
        for b in range(3):
            off = (r * 3 + b) * 34
            h = oracle_lib.float_to_half(scales[r])
            payload[off], payload[off + 1] = h & 0xFF, h >> 8
            for j in range(32):
                q = (r * 32 + b * 17 + j * 7) % 256 - 128
                payload[off + 2 + j] = q & 0xFF
                ref[r] += scales[r] * q * float(x[b * 32 + j])
    y = oracle_lib.q_matvec(payload, rows, cols, 0, x, order="scalar")
    assert np.all(np.abs(y - ref) <= 0.001)


def test_q4_all_nibbles_match_fp64(oracle_lib):
    """Q4Tests.AllNibblesBothHalvesAndSignedScalesMatchIndependentFp64 (Q4Tests.cs:8-37)."""
    rows, cols = 6, 96
    scales = [0.5, -2.0, 0.0, -0.0, 5.960464477539063e-08, 65504.0]
    x = np.array([(i % 17 - 8) / 32.0 for i in range(96)], np.float32)
    payload = np.zeros(rows * 3 * 18, np.uint8)
    ref = np.zeros(rows)
    for r in range(rows):
        for b in range(3):
            off = (r * 3 + b) * 18
            h = oracle_lib.float_to_half(scales[r])
            payload[off], payload[off + 1] = h & 0xFF, h >> 8
            for j in range(16):
                lo, hi = (j + b) % 16, (15 - j + b) % 16
                payload[off + 2 + j] = lo | (hi << 4)
                ref[r] += scales[r] * (lo - 8) * float(x[b * 32 + j])
                ref[r] += scales[r] * (hi - 8) * float(x[b * 32 + j + 16])
    for order in ("scalar", "avx2", "batch"):
        y = oracle_lib.q_matvec(payload, rows, cols, 1, x, order=order)
        assert np.all(np.abs(y - ref) <= 0.001), order


@pytest.mark.parametrize("fmt", [0, 1])
def test_q_avx2_bound_random(oracle_lib, fmt):
    """QuantizedAvx2Tests.SimdOrFallbackMatchesIndependentFp64AndDoesNotAllocate (:9-50)."""
    rng = np.random.default_rng(1729)
    for cols in (32, 64, 96, 288, 768):
        rows = 7
        bb = 34 if fmt == 0 else 18
        payload = rng.integers(0, 256, size=rows * (cols // 32) * bb, dtype=np.uint8)
        scales = [0.0, -0.0, 5.960464477539063e-08, 65504.0]
        for r in range(rows):
            for b in range(cols // 32):
                off = (r * (cols // 32) + b) * bb
                s = scales[r] if r < 4 else float(rng.random() * 4 - 2)
                h = oracle_lib.float_to_half(s)
                payload[off], payload[off + 1] = h & 0xFF, h >> 8
        x = (rng.random(cols) * 2 - 1).astype(np.float32)
        exact, mag = q_reference_fp64(payload, rows, cols, fmt, x)
        for order in ("avx2", "batch", "scalar"):
            y = oracle_lib.q_matvec(payload, rows, cols, fmt, x, order=order)
            assert np.all(np.abs(y - exact) <= gamma_bound(cols, mag)), (cols, order)


@pytest.mark.parametrize("fmt", [0, 1])
def test_intrinsic_orders_equal_scalar_emulation(oracle_lib, fmt):
    """The AVX2/FMA intrinsic restatements equal their lane-by-lane emulation bit for bit."""
    rng = np.random.default_rng(7)
    rows, cols = 33, 1024
    w = rng.standard_normal(rows * cols).astype(np.float32) * 0.02
    payload = oracle_lib.q_quantize(w, rows, cols, fmt)
    x = rng.standard_normal(cols * 3).astype(np.float32)
    assert bits_equal(oracle_lib.q_matvec(payload, rows, cols, fmt, x[:cols], order="avx2", threads=4),
                      oracle_lib.q_matvec(payload, rows, cols, fmt, x[:cols], order="avx2_emulated"))
    assert bits_equal(oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch", positions=3, threads=3),
                      oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch_emulated", positions=3))


# ----------------------------------------------------------------- Ternary2
def test_ternary2_encoding_kat(oracle_lib):
    """Ternary2Tests.EncodingMatchesIndependentBinaryFixture (Ternary2Tests.cs:9-22)."""
    kat = golden()["ternary2_encoding_kat"]
    w = np.zeros(64, np.float32)
    w[0], w[1] = 2.0, -2.0
    assert oracle_lib.t2_quantize(w, 1, 64, 64).tobytes().hex() == kat["expected_hex"]


def test_stq2_header_kat_and_corruptions(oracle_lib):
    """MappedTernary2Tests.RejectsInvalidHeaderLengthAndPayloadBeforeExecuting (:32-69)."""
    kat = golden()["stq2_header_kat"]
    payload = oracle_lib.t2_quantize(np.array([1.0], np.float32), 1, 1, 64)
    header = oracle_lib.stq2_header(1, 1, 64)
    assert header.hex() == kat["expected_hex"]
    original = header + payload.tobytes()
    assert oracle_lib.stq2_read_header(original) == (1, 1, 64)
    corruptions = [original[:10], original[:-1], original + b"\x00"]
    for index in (0, 4, 6, 8, 16, 20, 24):
        c = bytearray(original)
        c[index] ^= 0xFF
        corruptions.append(bytes(c))
    bad_code, bad_pad, bad_scale = bytearray(original), bytearray(original), bytearray(original)
    bad_code[36] = 3
    bad_pad[36] |= 4
    bad_scale[32:36] = np.array([np.nan], np.float32).tobytes()
    for data in corruptions:
        ok = True
        try:
            r, c_, b = oracle_lib.stq2_read_header(data)
        except oracle_lib.OracleError:
            ok = False
        else:
            ok = oracle_lib.t2_validate(np.frombuffer(data[32:], np.uint8), r, c_, b) == 0
        assert not ok
    for data in (bad_code, bad_pad, bad_scale):
        r, c_, b = oracle_lib.stq2_read_header(bytes(data))
        assert oracle_lib.t2_validate(np.frombuffer(bytes(data[32:]), np.uint8), r, c_, b) != 0


def test_ternary2_import_rejects_corrupt_blocks(oracle_lib):
    """Ternary2Tests.ImportRejectsCorruptBlocks (Ternary2Tests.cs:24-42)."""
    payload = np.zeros(20, np.uint8)
    payload[0:4] = np.frombuffer(np.float32(1).tobytes(), np.uint8)
    payload[4] = 3
    assert oracle_lib.t2_validate(payload, 1, 1, 64) == oracle_lib.ERR_ARGUMENT
    payload[4] = 4
    assert oracle_lib.t2_validate(payload, 1, 1, 64) == oracle_lib.ERR_ARGUMENT
    payload[4] = 1
    payload[0:4] = 0
    assert oracle_lib.t2_validate(payload, 1, 1, 64) == oracle_lib.ERR_ARGUMENT
    payload[4] = 0
    for s in (np.nan, np.inf, -1.0, -0.0):
        payload[0:4] = np.frombuffer(np.float32(s).tobytes(), np.uint8)
        assert oracle_lib.t2_validate(payload, 1, 1, 64) == oracle_lib.ERR_ARGUMENT


def test_ternary2_extreme_quantization(oracle_lib):
    """Ternary2Tests.QuantizationHandlesExtremeFiniteValuesAndRejectsNonFiniteValues (:90-102)."""
    for v in (FLT_MAX, 1.401298464324817e-45, 0.0):
        p = oracle_lib.t2_quantize(np.array([v, -v], np.float32), 1, 2, 64)
        np.testing.assert_array_equal(oracle_lib.t2_dequantize(p, 1, 2, 64), np.array([v, -v], np.float32))
    for v in (np.nan, np.inf, -np.inf):
        with pytest.raises(oracle_lib.OracleError):
            oracle_lib.t2_quantize(np.array([v], np.float32), 1, 1, 64)


@pytest.mark.parametrize("bs", [64, 128, 256])
def test_ternary2_critical_corpus_within_bound(oracle_lib, bs):
    """Ternary2Avx2Tests.VectorKernelMatchesReferenceIncludingTailsAndExtremeScales (:8-22) and the
    scalar twin; MappedTernary2Tests (:9-30) pins mapped == owned, which here is one code path."""
    cases = list(critical_cases(bs))
    for cols in list(range(1, 18)) + [63, 64, 65, 127, 128, 129, 255, 256, 257]:
        cases.append(numerical_random(3, cols))
    for name, rows, cols, w, x in cases:
        p = oracle_lib.t2_quantize(w, rows, cols, bs)
        assert oracle_lib.t2_validate(p, rows, cols, bs) == 0
        for order in ("avx2", "scalar"):
            y = oracle_lib.t2_matvec(p, rows, cols, bs, x, order=order)
            assert t2_bound_ok(p, rows, cols, bs, x, y), (name, cols, order)
        assert bits_equal(oracle_lib.t2_matvec(p, rows, cols, bs, x, order="avx2"),
                          oracle_lib.t2_matvec(p, rows, cols, bs, x, order="avx2_emulated")), (name, cols)


# ----------------------------------------------------------------- operators
def test_transformer_v1_operators(oracle_lib):
    """TransformerOpsTests.OperatorsMatchIndependentFloat64Fixtures (TransformerOpsTests.cs:8-25)."""
    g = golden()["transformer_v1"]
    x = np.array(g["x"], np.float32)
    assert operator_close(oracle_lib.rmsnorm(x, g["weights"], 1e-5), g["rms"])
    assert operator_close(oracle_lib.rope_interleaved(x, 48, 37), g["rope"])
    assert operator_close(oracle_lib.swiglu(g["gate"], g["up"]), g["swiglu"])
    out = oracle_lib.grouped_attention(g["query"], g["keys"], g["values"], 2, 2, 48, 7)
    assert operator_close(out, g["attention"])


def test_transformer_v2_operators(oracle_lib):
    """QwenOperatorTests (QwenOperatorTests.cs:28-94)."""
    g = golden()["transformer_v2"]
    a = g["gqa"]
    out = oracle_lib.grouped_attention(a["query"], a["keys"], a["values"], a["query_heads"], a["kv_heads"],
                                       a["head_dim"], a["tokens"])
    assert operator_close(out, a["output"])
    for key in ("rope_full", "rope_partial"):
        r = g[key]
        v = oracle_lib.rope_half(r["input"], r["head_dim"], r["position"], r["base"], r["rotary"])
        assert operator_close(v, r["output"]), key
    n = g["qk_norm"]
    assert operator_close(oracle_lib.rmsnorm_heads(n["input"], n["weights"], n["epsilon"], len(n["weights"])), n["output"])
    b = g["bias"]
    assert operator_close(oracle_lib.add(b["base"], b["bias"]), b["output"])


def test_attention_boundaries(oracle_lib):
    """fixtures/operators/attention-boundaries-v1.json (6 heads x 48, tokens 1..128)."""
    q, k, v = attention_boundary_inputs()
    for case in golden()["attention_boundaries_v1"]["cases"]:
        t = case["count"]
        out = oracle_lib.grouped_attention(q, k[:t].ravel(), v[:t].ravel(), 6, 6, 48, t)
        assert operator_close(out, case["expected"]), t


def test_extreme_operator_values(oracle_lib):
    """TransformerOpsTests.ExtremeFiniteValuesRemainStableAndInPlaceIsSafe (:27-42)."""
    x = np.array([FLT_MAX, -FLT_MAX], np.float32)
    np.testing.assert_array_equal(oracle_lib.rmsnorm(x, [1, 1], 1e-5), np.array([1, -1], np.float32))
    q = np.array([FLT_MAX, FLT_MAX], np.float32)
    k = np.array([FLT_MAX, FLT_MAX, -FLT_MAX, -FLT_MAX], np.float32)
    out = oracle_lib.grouped_attention(q, k, np.array([3, 4, 100, 200], np.float32), 1, 1, 2, 2)
    np.testing.assert_array_equal(out, np.array([3, 4], np.float32))


def test_gqa_equal_heads_is_mha_bitwise(oracle_lib):
    """QwenOperatorTests.GroupedQueryAttentionReducesToPlainAttentionWhenHeadsEqual (:45-60)."""
    rng = np.random.default_rng(11)
    q, k, v = (rng.random(n).astype(np.float32) for n in (8, 24, 24))
    a = oracle_lib.grouped_attention(q, k, v, 2, 2, 4, 3)
    b = oracle_lib.grouped_attention(q, k, v, 2, 2, 4, 3, threads=2)
    assert bits_equal(a, b)


def test_greedy_selector(oracle_lib):
    """GreedyTokenSelector.Select (GreedyTokenSelector.cs:6-16): smallest index of the maximum."""
    assert oracle_lib.greedy_select([1.0, 3.0, 3.0, -1.0]) == 1
    with pytest.raises(oracle_lib.OracleError):
        oracle_lib.greedy_select([1.0, np.nan])


# ---------------------------------------------------------------- K-quants (Q4_K, Q6_K, Q8_K)
def _kq():
    return golden()["kquants"]


def _close(actual, reference, abs_tol, rel_tol):
    return abs(float(actual) - reference) <= abs_tol + rel_tol * abs(reference)


@pytest.mark.parametrize("name,fmt", [("q4k_v1", 12), ("q6k_v1", 14)])
def test_k_decode_and_dot_match_reference(oracle_lib, name, fmt):
    """Q4KCodecTests / Q6KCodecTests (DecodedWeightsMatchReference, DotMatchesReference): the independent
    FP64 decode within 1e-3 + 1e-4 |w| and the scalar dot within 1e-2 + 1e-4 |dot|."""
    for case in _kq()[name]["cases"]:
        block = bytes.fromhex(case["block_hex"])
        w = oracle_lib.k_decode_row(block, 256, fmt)
        for a, r in zip(w, case["weights"]):
            assert _close(a, r, 1e-3, 1e-4), (case["name"], a, r)
        x = np.array(case["input"], np.float32)
        y = oracle_lib.k_matvec(block, 1, 256, fmt, x, order="scalar")
        assert _close(y[0], case["dot"], 1e-2, 1e-4), (case["name"], y[0], case["dot"])
        y2 = oracle_lib.k_matvec(block, 1, 256, fmt, x, order="avx2")
        assert _close(y2[0], case["dot"], 1e-2, 1e-4), (case["name"], "avx2")


def test_zero_q4k_block_decodes_to_zeros(oracle_lib):
    zero = next(c for c in _kq()["q4k_v1"]["cases"] if c["name"] == "zero")
    assert np.all(oracle_lib.k_decode_row(bytes.fromhex(zero["block_hex"]), 256, 12) == 0)


def test_q8k_quantizer_bytes_and_q4k_integer_product(oracle_lib):
    """Q8KCodecTests (QuantizerMatchesTheReferenceBytes, ScaleAndGroupSums, IntegerProductMatchesTheReferenceDot):
    the quantized block equals ggml's bytes exactly; the Q4_K x Q8_K product within 1e-3 + 1e-4 |dot|."""
    import struct
    for case in _kq()["q8k_v1"]["cases"]:
        x = np.array(case["input"], np.float32)
        q = oracle_lib.q8k_quantize_row(x)
        assert q.tobytes() == bytes.fromhex(case["block_hex"]), case["name"]
        assert list(q[4:260].view(np.int8)) == case["codes"]
        assert list(q[260:292].view(np.int16)) == case["bsums"]
        scale = struct.unpack("<f", q[:4].tobytes())[0]
        assert abs(scale - case["scale"]) <= 1e-6 * max(1.0, abs(case["scale"]))
        w = bytes.fromhex(case["weights_hex"])
        dot, mins = oracle_lib.k_int_dot(w, 12, q)
        d = oracle_lib.half_to_float(w[0] | (w[1] << 8))
        dmin = oracle_lib.half_to_float(w[2] | (w[3] << 8))
        value = np.float32(np.float32(d) * np.float32(scale)) * np.float32(dot) - \
            np.float32(np.float32(dmin) * np.float32(scale)) * np.float32(mins)
        assert _close(value, case["dot"], 1e-3, 1e-4), case["name"]


def test_q6k_integer_product(oracle_lib):
    """Q6KQuantizedProductTests.IntegerProductMatchesTheIndependentReference and the decoder composition."""
    import struct
    cases = _kq()["q6k_q8k_v1"]["cases"]
    assert len(cases) == 5
    for case in cases:
        w = bytes.fromhex(case["weights_hex"])
        a = bytes.fromhex(case["activation_hex"])
        scale = struct.unpack("<f", a[:4])[0]
        dot, _ = oracle_lib.k_int_dot(w, 14, a)
        d = oracle_lib.half_to_float(w[208] | (w[209] << 8))
        value = np.float32(np.float32(scale) * np.float32(d)) * np.float32(dot)
        assert _close(value, case["dot"], 1e-3, 1e-4), case["name"]
        decoded = oracle_lib.k_decode_row(w, 256, 14).astype(np.float64)
        codes = np.frombuffer(a[4:260], np.int8).astype(np.float64)
        assert _close(value, float(decoded @ codes) * scale, 1e-3, 1e-4)


def test_real_tensor_blocks(oracle_lib):
    """KParityTests.RealTensorBlocksDecodeToTheIndependentReference: blocks of a real Q4_K_M model."""
    for case in _kq()["k_real_v1"]["cases"]:
        fmt = 12 if case["name"].startswith("q4k:") else 14
        raw = bytes.fromhex(case["block_hex"])
        w = oracle_lib.k_decode_row(raw, 256 * case["blocks"], fmt)
        for a, r in zip(w, case["weights"]):
            assert _close(a, r, 1e-3, 1e-4), case["name"]
        x = np.array(case["input"], np.float32)
        bb = 144 if fmt == 12 else 210
        for b in range(case["blocks"]):
            y = oracle_lib.k_matvec(raw[b * bb:(b + 1) * bb], 1, 256, fmt, x, order="scalar")
            assert _close(y[0], case["dots"][b], 1e-2, 1e-4), (case["name"], b)


@pytest.mark.parametrize("cols,threads", [(3584, 1), (18944, 8)])
def test_q4k_batch_matches_block_products(oracle_lib, cols, threads):
    """KParityTests.Q4DecodeMatchesThePublicQuantizedCodecs: the batched integer path equals the per-block
    quantized products (17 rows cycling the fixture blocks, sin input)."""
    blocks_hex = [bytes.fromhex(c["block_hex"]) for c in _kq()["q4k_v1"]["cases"]]
    rows, nb = 17, cols // 256
    payload = b"".join(blocks_hex[(r + b) % len(blocks_hex)] for r in range(rows) for b in range(nb))
    x = np.sin(np.arange(cols) * 0.017).astype(np.float32)
    got = oracle_lib.k_matvec(payload, rows, cols, 12, x, order="batch", threads=threads)
    act = oracle_lib.q8k_quantize_row(x)
    import struct
    for r in range(rows):
        expected = 0.0
        for b in range(nb):
            a = act[b * 292:(b + 1) * 292]
            s = struct.unpack("<f", a[:4].tobytes())[0]
            blk = payload[(r * nb + b) * 144:(r * nb + b + 1) * 144]
            dot, mins = oracle_lib.k_int_dot(blk, 12, a)
            d = oracle_lib.half_to_float(blk[0] | (blk[1] << 8))
            dm = oracle_lib.half_to_float(blk[2] | (blk[3] << 8))
            expected += float(np.float32(np.float32(d) * np.float32(s)) * np.float32(dot)
                              - np.float32(np.float32(dm) * np.float32(s)) * np.float32(mins))
        assert _close(got[r], expected, 1e-3, 1e-5), r


def test_k_validation(oracle_lib):
    """Q4KCodecTests / Q6KCodecTests.NonFiniteSuperBlockScaleIsRejected and the shape rule."""
    p = np.zeros(144, np.uint8)
    p[1] = 0x7C
    assert oracle_lib.k_validate(p, 1, 256, 12) == oracle_lib.ERR_INVALID_DATA
    p = np.zeros(144, np.uint8)
    p[3] = 0x7C
    assert oracle_lib.k_validate(p, 1, 256, 12) == oracle_lib.ERR_INVALID_DATA
    p = np.zeros(210, np.uint8)
    p[209] = 0x7C
    assert oracle_lib.k_validate(p, 1, 256, 14) == oracle_lib.ERR_INVALID_DATA
    assert oracle_lib.k_validate(np.zeros(210, np.uint8), 1, 256, 14) == oracle_lib.OK
    with pytest.raises(oracle_lib.OracleError):
        oracle_lib.k_geometry(1, 128, 14)


# ---------------------------------------------------------------- ternary bitplane (STB1)
def _tb_kat():
    p = np.zeros(20, np.uint8)
    p[0:4] = np.frombuffer(np.float32(0.5).tobytes(), np.uint8)
    p[4], p[12] = 0x89, 0x14
    return p


def test_bitplane_golden_and_invalid_planes(oracle_lib):
    """TernaryBitplaneTests.IndependentGoldenAndCodecRejectInvalidPlanes and docs/ternary-bitplane-v1.md's
    example: scale 0.5, codes [+1,0,-1,+1,-1,0,0,+1] -> P 0x89, N 0x14; ones -> 0.5; Ternary2 bytes 61 42."""
    p = _tb_kat()
    assert oracle_lib.tb_validate(p, 1, 8, 64) == oracle_lib.OK
    ones = np.ones(8, np.float32)
    assert oracle_lib.tb_matvec(p, 1, 8, 64, ones, "scalar")[0] == 0.5
    assert oracle_lib.tb_matvec(p, 1, 8, 64, ones, "avx2")[0] == 0.5
    t2 = oracle_lib.tb_to_t2(p, 1, 8, 64)
    assert (t2[4], t2[5]) == (0x61, 0x42)
    assert np.array_equal(oracle_lib.tb_from_t2(t2, 1, 8, 64), p)
    for defect in range(5):
        bad = p.copy()
        if defect == 0:
            bad[12] |= 1
        elif defect == 1:
            bad[5] = 1
        else:
            bad[0:4] = np.frombuffer(np.float32([-0.0, np.nan, 0.0][defect - 2]).tobytes(), np.uint8)
        assert oracle_lib.tb_validate(bad, 1, 8, 64) == oracle_lib.ERR_ARGUMENT, defect


@pytest.mark.parametrize("bs", [64, 128, 256])
def test_bitplane_round_trip_and_scalar_parity(oracle_lib, bs):
    """TernaryBitplaneTests.CorpusRoundTripPreservesEveryByteAndScalarResult: Ternary2 -> bitplane -> Ternary2
    is byte-identical; the bitplane scalar MatVec equals the Ternary2 scalar MatVec; the bitplane AVX2 kernel
    equals the Ternary2 AVX2 kernel (same logical codes, same lane arithmetic)."""
    for name, rows, cols, w, x in list(critical_cases(bs)) + [numerical_random(3, c) for c in (1, 17, 257, 1000)]:
        t2 = oracle_lib.t2_quantize(w, rows, cols, bs)
        tb = oracle_lib.tb_from_t2(t2, rows, cols, bs)
        assert oracle_lib.tb_validate(tb, rows, cols, bs) == oracle_lib.OK
        assert np.array_equal(oracle_lib.tb_to_t2(tb, rows, cols, bs), t2), name
        assert bits_equal(oracle_lib.tb_matvec(tb, rows, cols, bs, x, "scalar"),
                          oracle_lib.t2_matvec(t2, rows, cols, bs, x, "scalar")), name
        assert bits_equal(oracle_lib.tb_matvec(tb, rows, cols, bs, x, "avx2"),
                          oracle_lib.t2_matvec(t2, rows, cols, bs, x, "avx2")), name
