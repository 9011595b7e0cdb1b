"""The ternary bitplane layout (STB1, docs/ternary-bitplane-v1.md) on the GPU through the C ABI, against the
oracle's restatement of TernaryBitplaneMatVec / TernaryBitplaneAvx2Kernel, bit for bit; the lossless
Ternary2 round trip; the reference's golden block, rejections and file checks
(tests/Satori.Numerics.Tests/TernaryBitplaneTests.cs)."""
import numpy as np
import pytest

from golden_util import bits_equal, critical_cases, numerical_random, seeded_normal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sat():
    from satori_b200 import build
    build.build()
    import satori_b200
    return satori_b200


@pytest.fixture(scope="module")
def ctx(sat):
    return sat.default_context(0)


def _golden_payload():
    p = np.zeros(20, np.uint8)
    p[0:4] = np.frombuffer(np.float32(0.5).tobytes(), np.uint8)
    p[4], p[12] = 0x89, 0x14
    return p


def test_golden_block_and_invalid_planes(sat, ctx):
    m = sat.TernaryBitplaneMatrix.from_packed(1, 8, 64, _golden_payload(), ctx=ctx)
    ones = np.ones(8, np.float32)
    assert sat.TernaryBitplaneMatVec.execute_scalar(m, ones)[0] == 0.5
    assert sat.TernaryBitplaneMatVec.execute(m, ones)[0] == 0.5
    t2 = m.to_ternary2().data
    assert (t2[4], t2[5]) == (0x61, 0x42)
    for defect in range(5):
        bad = _golden_payload()
        if defect == 0:
            bad[12] |= 1
        elif defect == 1:
            bad[5] = 1
        else:
            bad[0:4] = np.frombuffer(np.float32([-0.0, np.nan, 0.0][defect - 2]).tobytes(), np.uint8)
        with pytest.raises(sat.ArgumentError):
            sat.TernaryBitplaneMatrix.from_packed(1, 8, 64, bad, ctx=ctx)


@pytest.mark.parametrize("bs", [64, 128, 256])
def test_corpus_round_trip_and_both_orders(sat, ctx, oracle_lib, bs):
    cases = list(critical_cases(bs)) + [numerical_random(3, c) for c in (17, 257, 1000)]
    for name, rows, cols, w, x in cases:
        t2 = sat.Ternary2Matrix.quantize(w, rows, cols, bs, ctx=ctx)
        tb = sat.TernaryBitplaneMatrix.from_ternary2(t2)
        assert np.array_equal(tb.data, oracle_lib.tb_from_t2(t2.data, rows, cols, bs)), name
        assert np.array_equal(tb.to_ternary2().data, t2.data), name
        assert bits_equal(sat.TernaryBitplaneMatVec.execute_scalar(tb, x),
                          oracle_lib.tb_matvec(tb.data, rows, cols, bs, x, "scalar")), (name, "scalar")
        assert bits_equal(sat.TernaryBitplaneMatVec.execute(tb, x),
                          oracle_lib.tb_matvec(tb.data, rows, cols, bs, x, "avx2")), (name, "avx2")
        dec = np.stack([tb.device.read_row(r) for r in range(rows)]).reshape(-1)
        assert bits_equal(dec, oracle_lib.t2_dequantize(t2.data, rows, cols, bs)), name


@pytest.mark.parametrize("bs", [64, 128, 256])
@pytest.mark.parametrize("n", [1024, 4096])
def test_benchmark_shapes_stream_kernel(sat, ctx, oracle_lib, bs, n):
    """Whole blocks take the row-streaming kernel, for both layouts; both equal the AVX2-order oracle."""
    w = seeded_normal(300 + n + bs, n * n)
    x = seeded_normal(400 + n, n)
    t2 = sat.Ternary2Matrix.quantize(w, n, n, bs, ctx=ctx)
    tb = sat.TernaryBitplaneMatrix.from_ternary2(t2)
    ref = oracle_lib.tb_matvec(tb.data, n, n, bs, x, "avx2")
    assert bits_equal(sat.TernaryBitplaneMatVec.execute(tb, x), ref)
    assert bits_equal(sat.Ternary2MatVec.execute(t2, x), ref)


def test_file_header_and_truncations(sat, ctx, tmp_path):
    m = sat.TernaryBitplaneMatrix.from_packed(1, 8, 64, _golden_payload(), ctx=ctx)
    path = str(tmp_path / "m.stb1")
    m.save(path)
    raw = open(path, "rb").read()
    assert raw[:4] == b"STB1" and raw[4:6] == b"\x01\x00" and int.from_bytes(raw[24:32], "little") == 20
    assert np.array_equal(sat.TernaryBitplaneMatrix.load(path, ctx=ctx).data, _golden_payload())
    for length in range(len(raw)):
        p = str(tmp_path / f"t{length}.stb1")
        open(p, "wb").write(raw[:length])
        with pytest.raises(sat.InvalidDataError):
            sat.TernaryBitplaneMatrix.load(p, ctx=ctx)
