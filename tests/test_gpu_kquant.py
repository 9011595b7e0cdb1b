"""GGUF K-quant matrices (Q4_K, Q6_K) on the GPU through the C ABI, against the oracle, bit for bit, in
all three orders: batch (QuantizedMatVec.ExecuteBatch -> Q8_K activations and exact integer products,
what decode runs), scalar (ExecuteScalar -> Q4KCodec/Q6KCodec.DotBlock) and execute
(QuantizedKAvx2Kernel.ExecuteQ4K/Q6K), plus row decode and the non-finite scale rejection."""
import numpy as np
import pytest

from golden_util import bits_equal, golden

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


def _exact(gpu, ref, what):
    gpu, ref = np.asarray(gpu, np.float32), np.asarray(ref, np.float32)
    assert bits_equal(gpu, ref), (what, np.flatnonzero(gpu.view(np.uint32) != ref.view(np.uint32))[:8],
                                  gpu[:4], ref[:4])


def _random_k(rng, rows, cols, fmt):
    bb = 144 if fmt == 12 else 210
    p = rng.integers(0, 256, size=rows * (cols // 256) * bb, dtype=np.uint8).reshape(-1, bb)
    scales = (rng.standard_normal((p.shape[0], 2)) * 0.01).astype(np.float16).view(np.uint16)
    if fmt == 12:
        p[:, 0], p[:, 1] = scales[:, 0] & 0xFF, scales[:, 0] >> 8
        p[:, 2], p[:, 3] = scales[:, 1] & 0xFF, scales[:, 1] >> 8
    else:
        p[:, 208], p[:, 209] = scales[:, 0] & 0xFF, scales[:, 0] >> 8
    return p.reshape(-1)


@pytest.mark.parametrize("name,fmt", [("q4k_v1", 12), ("q6k_v1", 14)])
def test_fixture_blocks_all_orders(sat, ctx, oracle_lib, name, fmt):
    for case in golden()["kquants"][name]["cases"]:
        block = np.frombuffer(bytes.fromhex(case["block_hex"]), np.uint8)
        x = np.array(case["input"], np.float32)
        m = sat.CudaMatrixFactory(ctx).create(block, sat.QuantizedMatrixShape(1, 256, fmt))
        _exact(m.read_row(0), oracle_lib.k_decode_row(block, 256, fmt), (case["name"], "decode"))
        _exact(m.execute_scalar(x), oracle_lib.k_matvec(block, 1, 256, fmt, x, "scalar"), (case["name"], "scalar"))
        _exact(m.execute(x), oracle_lib.k_matvec(block, 1, 256, fmt, x, "avx2"), (case["name"], "execute"))
        _exact(m.execute_batch(x, 1), oracle_lib.k_matvec(block, 1, 256, fmt, x, "batch"), (case["name"], "batch"))
        m.dispose()


@pytest.mark.parametrize("fmt", [12, 14])
@pytest.mark.parametrize("rows,cols,positions", [(37, 256, 1), (64, 3584, 3), (300, 18944, 1), (9, 4096, 2)])
def test_random_payloads_bit_exact(sat, ctx, oracle_lib, fmt, rows, cols, positions):
    rng = np.random.default_rng(rows + cols + fmt)
    payload = _random_k(rng, rows, cols, fmt)
    x = rng.standard_normal(positions * cols).astype(np.float32)
    x[:256] = 0.0 if cols > 256 else x[:256]          # an all-zero activation block is skipped
    m = sat.CudaMatrixFactory(ctx).create(payload, sat.QuantizedMatrixShape(rows, cols, fmt))
    _exact(m.execute_batch(x, positions),
           oracle_lib.k_matvec(payload, rows, cols, fmt, x, "batch", positions=positions, threads=8), "batch")
    if rows * cols <= 64 * 4096:
        _exact(m.execute_scalar(x[:cols]), oracle_lib.k_matvec(payload, rows, cols, fmt, x[:cols], "scalar"), "scalar")
        _exact(m.execute(x[:cols]), oracle_lib.k_matvec(payload, rows, cols, fmt, x[:cols], "avx2", threads=8), "execute")
    for r in (0, rows - 1):
        bb = 144 if fmt == 12 else 210
        row = payload[r * (cols // 256) * bb:(r + 1) * (cols // 256) * bb]
        _exact(m.read_row(r), oracle_lib.k_decode_row(row, cols, fmt), ("row", r))
    m.dispose()


def test_k_real_tensor_blocks(sat, ctx, oracle_lib):
    """Blocks of the reference's real Q4_K_M tensors (k-real-v1): decode and scalar dot bitwise."""
    for case in golden()["kquants"]["k_real_v1"]["cases"]:
        fmt = 12 if case["name"].startswith("q4k:") else 14
        raw = np.frombuffer(bytes.fromhex(case["block_hex"]), np.uint8)
        cols = 256 * case["blocks"]
        m = sat.CudaMatrixFactory(ctx).create(raw, sat.QuantizedMatrixShape(1, cols, fmt))
        _exact(m.read_row(0), oracle_lib.k_decode_row(raw, cols, fmt), case["name"])
        x = np.tile(np.array(case["input"], np.float32), case["blocks"])
        _exact(m.execute_batch(x, 1), oracle_lib.k_matvec(raw, 1, cols, fmt, x, "batch"), case["name"])
        m.dispose()


@pytest.mark.parametrize("fmt,offset", [(12, 1), (12, 3), (14, 209)])
def test_nonfinite_super_block_scale_rejected(sat, ctx, fmt, offset):
    """Q4KCodecTests / Q6KCodecTests.NonFiniteSuperBlockScaleIsRejected."""
    p = np.zeros(144 if fmt == 12 else 210, np.uint8)
    p[offset] = 0x7C
    with pytest.raises(sat.InvalidDataError):
        sat.CudaMatrixFactory(ctx).create(p, sat.QuantizedMatrixShape(1, 256, fmt))
    with pytest.raises(sat.ArgumentError):
        sat.QuantizedMatrixShape(1, 128, fmt)
