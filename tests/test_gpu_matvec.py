"""GPU parity of the quantized MatVec (Q8_0, Q4_0, Ternary2 64/128/256) through the C ABI.

The CUDA kernels reproduce the reference's FP32 operation order, so every comparison with the
oracle is bit-exact (``bits_equal``; +0 and -0 compare equal).  The north_star tolerance
(1e-5 relative + 1e-6 absolute) is asserted as well, and is implied by bit-exactness.
"""
import numpy as np
import pytest

from golden_util import bits_equal, critical_cases, golden, north_star_close, numerical_random, q8_critical_cases, \
    seeded_normal

pytestmark = pytest.mark.gpu

ORDERS_Q = (("execute", "avx2"), ("execute_scalar", "scalar"), ("execute_batch", "batch"))


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


@pytest.fixture(scope="module")
def ctx(sat):
    return sat.default_context(0)


def _q_run(m, method, x, positions=1):
    if method == "execute_batch":
        return m.execute_batch(x, positions)
    return getattr(m, method)(x)


def _assert_exact(gpu, ref, what):
    gpu = np.asarray(gpu, np.float32)
    ref = np.asarray(ref, np.float32)
    assert bits_equal(gpu, ref), (what, np.flatnonzero(gpu.view(np.uint32) != ref.view(np.uint32))[:8])
    assert np.all(north_star_close(gpu, ref)), what


# ---------------------------------------------------------------- golden files
@pytest.mark.parametrize("name,fmt", [("q8_0", 0), ("q4_0", 1)])
def test_gguf_golden_through_gpu(sat, ctx, name, fmt):
    """QuantizedTests.cs:9-25 / QuantizedAvx2Tests.cs:52-65 on the GPU: ones . decode = -8 exactly."""
    g = golden()["gguf_v1"][name]
    payload = bytes.fromhex(g["payload_hex"])
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(1, 32, fmt))
    ones = np.ones(32, np.float32)
    for method, _ in ORDERS_Q:
        assert _q_run(m, method, ones)[0] == np.float32(-8.0), method
    if fmt == 0:
        np.testing.assert_array_equal(m.read_row(0), np.array(g["decoded_weights"], np.float32))
    else:
        with pytest.raises(sat.NotSupportedError):
            m.read_row(0)


@pytest.mark.parametrize("bits", [0x7C00, 0xFC00, 0x7E00])
@pytest.mark.parametrize("fmt", [0, 1])
def test_nonfinite_scale_rejected_at_create(sat, ctx, bits, fmt):
    payload = np.zeros(34 if fmt == 0 else 18, np.uint8)
    payload[0], payload[1] = bits & 0xFF, bits >> 8
    with pytest.raises(sat.InvalidDataError):
        sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(1, 32, fmt))


# ---------------------------------------------------------------- Q8_0 / Q4_0 parity
def test_q8_critical_cases_bit_exact(sat, ctx, oracle_lib):
    """Q8Validation.CriticalCases (Q8Validation.cs:9-28): 30 shapes, signed/zero/subnormal/max scales."""
    for name, rows, cols, payload, x in q8_critical_cases():
        m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, 0))
        for method, order in ORDERS_Q:
            _assert_exact(_q_run(m, method, x), oracle_lib.q_matvec(payload, rows, cols, 0, x, order=order),
                          (name, method))
        m.dispose()


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (63, 288), (129, 768), (33, 1536), (300, 4096)])
def test_random_payloads_bit_exact(sat, ctx, oracle_lib, fmt, rows, cols):
    """Random bytes (every code value) with finite random scales, all three orders."""
    rng = np.random.default_rng(rows * 1000 + cols + fmt)
    bb = 34 if fmt == 0 else 18
    payload = rng.integers(0, 256, size=rows * (cols // 32) * bb, dtype=np.uint8)
    scales = (rng.standard_normal(rows * (cols // 32)) * 0.05).astype(np.float16).view(np.uint16)
    p2 = payload.reshape(-1, bb)
    p2[:, 0] = scales & 0xFF
    p2[:, 1] = scales >> 8
    x = rng.standard_normal(cols).astype(np.float32)
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
    for method, order in ORDERS_Q:
        _assert_exact(_q_run(m, method, x), oracle_lib.q_matvec(payload, rows, cols, fmt, x, order=order), method)


@pytest.mark.parametrize("fmt,rows,cols", [(0, 4096, 4096), (1, 11008, 4096), (1, 3584, 18944), (0, 8960, 1536)])
def test_baseline_shapes_bit_exact(sat, ctx, oracle_lib, fmt, rows, cols):
    """BASELINE config 2 shapes (and two decode projections): seeded N(0, 0.02^2) weights, N(0,1) input."""
    w = seeded_normal(11 + fmt, rows * cols, 0.02)
    payload = oracle_lib.q_quantize(w, rows, cols, fmt)
    x = seeded_normal(12 + fmt, cols)
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
    _assert_exact(m.execute_batch(x, 1), oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch", threads=8),
                  "batch")
    _assert_exact(m.execute(x), oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="avx2", threads=8), "execute")


@pytest.mark.parametrize("fmt,rows,cols", [(0, 3, 8448), (1, 500, 8960), (0, 1536, 8960), (1, 37, 12288),
                                           (0, 61, 12544), (1, 3584, 18944), (0, 100, 24576), (1, 29, 24832)])
def test_decode_order_row_widths_bit_exact(sat, ctx, oracle_lib, fmt, rows, cols):
    """ExecuteBatch at one position across the widths that pick each decode kernel shape (one or two
    block columns per lane, 8 or 12 compute warps, and the column-chunked kernel past 24576)."""
    rng = np.random.default_rng(rows + cols + fmt)
    bb = 34 if fmt == 0 else 18
    payload = rng.integers(0, 256, size=rows * (cols // 32) * bb, dtype=np.uint8)
    scales = (rng.standard_normal(rows * (cols // 32)) * 0.05).astype(np.float16).view(np.uint16)
    p2 = payload.reshape(-1, bb)
    p2[:, 0] = scales & 0xFF
    p2[:, 1] = scales >> 8
    x = rng.standard_normal(cols).astype(np.float32)
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
    _assert_exact(m.execute_batch(x, 1), oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch", threads=8),
                  "batch")


@pytest.mark.parametrize("cols", [1536, 3584, 4096, 8960, 18944])
@pytest.mark.parametrize("fmt", [0, 1])
def test_fixed_width_stream_kernel_bit_exact(sat, ctx, oracle_lib, fmt, cols):
    """The decode configurations' row widths take gemv_stream (width fixed at compile time): one row,
    a row count that leaves partial stages and fold batches, and one that spans every CTA."""
    bb = 34 if fmt == 0 else 18
    for rows in (1, 37, 1003):
        rng = np.random.default_rng(rows * 7 + cols + fmt)
        payload = rng.integers(0, 256, size=rows * (cols // 32) * bb, dtype=np.uint8)
        scales = (rng.standard_normal(rows * (cols // 32)) * 0.05).astype(np.float16).view(np.uint16)
        p2 = payload.reshape(-1, bb)
        p2[:, 0] = scales & 0xFF
        p2[:, 1] = scales >> 8
        x = rng.standard_normal(cols).astype(np.float32)
        m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
        _assert_exact(m.execute_batch(x, 1),
                      oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch", threads=8), ("batch", rows))
        m.dispose()


@pytest.mark.parametrize("positions", [2, 3, 8, 11])
def test_batch_positions_bit_exact(sat, ctx, oracle_lib, positions):
    """ExecuteBatch with several positions: each position's rows equal the reference's."""
    rows, cols = 257, 1024
    for fmt in (0, 1):
        w = seeded_normal(5, rows * cols, 0.02)
        payload = oracle_lib.q_quantize(w, rows, cols, fmt)
        x = seeded_normal(6, positions * cols)
        m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
        _assert_exact(m.execute_batch(x, positions),
                      oracle_lib.q_matvec(payload, rows, cols, fmt, x, order="batch", positions=positions), fmt)


def test_read_row_bit_exact_and_output_untouched_on_error(sat, ctx, oracle_lib):
    rows, cols = 64, 1536
    payload = oracle_lib.q_quantize(seeded_normal(3, rows * cols), rows, cols, 0)
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, 0))
    rb = cols // 32 * 34
    for r in (0, 17, 63):
        np.testing.assert_array_equal(m.read_row(r), oracle_lib.q_decode_row(payload[r * rb:(r + 1) * rb], cols, 0))
    out = np.full(rows, 7.0, np.float32)
    with pytest.raises(sat.ArgumentError):
        m.execute(np.ones(cols + 1, np.float32), out)
    assert np.all(out == 7.0)
    m.dispose()
    with pytest.raises(sat.DisposedError):
        m.execute(np.ones(cols, np.float32))


# ---------------------------------------------------------------- Ternary2 parity
@pytest.mark.parametrize("bs", [64, 128, 256])
def test_ternary2_critical_corpus_bit_exact(sat, ctx, oracle_lib, bs):
    """Ternary2Avx2Tests.cs:8-22 corpus + columns 1..17, 63-65, 127-129, 255-257 (tails), both orders."""
    cases = list(critical_cases(bs))
    for cols in list(range(1, 18)) + [63, 64, 65, 127, 128, 129, 255, 256, 257]:
        cases.append(numerical_random(3, cols))
    for name, rows, cols, w, x in cases:
        m = sat.Ternary2Matrix.quantize(w, rows, cols, bs, ctx=ctx)
        ref_payload = oracle_lib.t2_quantize(w, rows, cols, bs)
        np.testing.assert_array_equal(m.data, ref_payload, err_msg=f"quantize {name} {cols}")
        _assert_exact(sat.Ternary2MatVec.execute(m, x), oracle_lib.t2_matvec(ref_payload, rows, cols, bs, x, "avx2"),
                      (name, cols, "avx2"))
        _assert_exact(sat.Ternary2MatVec.execute_scalar(m, x),
                      oracle_lib.t2_matvec(ref_payload, rows, cols, bs, x, "scalar"), (name, cols, "scalar"))
        np.testing.assert_array_equal(m.dequantize(), oracle_lib.t2_dequantize(ref_payload, rows, cols, bs))


@pytest.mark.parametrize("bs", [64, 128, 256])
@pytest.mark.parametrize("n", [1024, 2048, 4096])
def test_ternary2_benchmark_shapes_bit_exact(sat, ctx, oracle_lib, bs, n):
    """n x n, N(0,1) weights quantized with absmean scales, N(0,1) input."""
    w = seeded_normal(100 + n + bs, n * n)
    x = seeded_normal(200 + n, n)
    m = sat.Ternary2Matrix.quantize(w, n, n, bs, ctx=ctx)
    ref = oracle_lib.t2_quantize(w, n, n, bs)
    np.testing.assert_array_equal(m.data, ref)
    _assert_exact(sat.Ternary2MatVec.execute(m, x), oracle_lib.t2_matvec(ref, n, n, bs, x, "avx2", threads=8), "avx2")
    if n <= 2048:
        _assert_exact(sat.Ternary2MatVec.execute_scalar(m, x), oracle_lib.t2_matvec(ref, n, n, bs, x, "scalar"),
                      "scalar")


def test_ternary2_import_rejections(sat, ctx):
    """Ternary2Tests.ImportRejectsCorruptBlocks (Ternary2Tests.cs:24-42)."""
    payload = np.zeros(20, np.uint8)
    payload[0:4] = np.frombuffer(np.float32(1).tobytes(), np.uint8)
    for code in (3, 4):  # invalid code; nonzero padding after the single valid weight
        p = payload.copy()
        p[4] = code
        with pytest.raises(sat.ArgumentError):
            sat.Ternary2Matrix.from_packed(1, 1, 64, p, ctx=ctx)
    p = payload.copy()
    p[4] = 1
    p[0:4] = 0
    with pytest.raises(sat.ArgumentError):
        sat.Ternary2Matrix.from_packed(1, 1, 64, p, ctx=ctx)
    for s in (np.nan, np.inf, -1.0, -0.0):
        p = payload.copy()
        p[0:4] = np.frombuffer(np.float32(s).tobytes(), np.uint8)
        with pytest.raises(sat.ArgumentError):
            sat.Ternary2Matrix.from_packed(1, 1, 64, p, ctx=ctx)


def test_native_stq2_reader_equals_owned_and_rejects_corruption(sat, ctx, tmp_path):
    """satori_stq2_open (MappedTernary2Matrix in native code): equal to the owned matrix bitwise, and the
    header / length / payload corruptions of MappedTernary2Tests.cs:32-69 raise InvalidDataError."""
    name, rows, cols, w, x = numerical_random(7, 257)
    owned = sat.Ternary2Matrix.quantize(w, rows, cols, 64, ctx=ctx)
    path = str(tmp_path / "m.stq2")
    owned.save(path)
    m = sat.open_stq2(path, ctx=ctx)
    assert (m.rows, m.columns, m.format) == (rows, cols, 64)
    assert bits_equal(m.execute(x), sat.Ternary2MatVec.execute(owned, x))
    m.dispose()
    one = sat.Ternary2Matrix.quantize(np.array([1.0], np.float32), 1, 1, 64, ctx=ctx)
    p1 = str(tmp_path / "one.stq2")
    one.save(p1)
    original = open(p1, "rb").read()
    corruptions = [original[:10], original[:-1], original + b"\x00"]
    for index in (0, 4, 6, 8, 16, 20, 24):
        c = bytearray(original)
        c[index] ^= 0xFF
        corruptions.append(bytes(c))
    for i, data in enumerate(corruptions):
        pc = str(tmp_path / f"n{i}.stq2")
        open(pc, "wb").write(data)
        with pytest.raises(sat.InvalidDataError):
            sat.open_stq2(pc, ctx=ctx)


def test_mapped_ternary2_equals_owned_and_rejects_corruption(sat, ctx, tmp_path):
    """MappedTernary2Tests.cs:9-30 (mapped == owned, bitwise), :32-69 (12 corruptions) and :71-89."""
    name, rows, cols, w, x = numerical_random(7, 257)
    owned = sat.Ternary2Matrix.quantize(w, rows, cols, 64, ctx=ctx)
    path = str(tmp_path / "m.stq2")
    owned.save(path)
    with sat.MappedTernary2Matrix(path, ctx=ctx) as mapped:
        assert bits_equal(mapped.execute(x), sat.Ternary2MatVec.execute(owned, x))
        assert bits_equal(mapped.execute_scalar(x), sat.Ternary2MatVec.execute_scalar(owned, x))
    mapped = sat.MappedTernary2Matrix(path, ctx=ctx)
    mapped.dispose()
    with pytest.raises(sat.DisposedError):
        mapped.execute(x)
    one = sat.Ternary2Matrix.quantize(np.array([1.0], np.float32), 1, 1, 64, ctx=ctx)
    p1 = str(tmp_path / "one.stq2")
    one.save(p1)
    original = open(p1, "rb").read()
    assert original[:32].hex() == golden()["stq2_header_kat"]["expected_hex"]
    corruptions = [original[:10], original[:-1], original + b"\x00"]
    for index in (0, 4, 6, 8, 16, 20, 24):
        c = bytearray(original)
        c[index] ^= 0xFF
        corruptions.append(bytes(c))
    for mutate in (lambda b: b.__setitem__(36, 3), lambda b: b.__setitem__(36, b[36] | 4),
                   lambda b: b.__setitem__(slice(32, 36), np.float32(np.nan).tobytes())):
        c = bytearray(original)
        mutate(c)
        corruptions.append(bytes(c))
    for i, data in enumerate(corruptions):
        pc = str(tmp_path / f"c{i}.stq2")
        open(pc, "wb").write(data)
        with pytest.raises(sat.InvalidDataError):
            sat.MappedTernary2Matrix(pc, ctx=ctx)
