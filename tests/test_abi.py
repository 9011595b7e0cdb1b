"""CPU-only checks of the C-ABI library and the host-side mirror (no GPU compute).

* the in-tree libsatori_cuda.so loads and exports every function include/satori_cuda.h declares;
* the Python mirror's host logic (shapes, STQ2 header codec) matches the reference's rules and KATs.
"""
import os
import subprocess

import pytest

from golden_util import golden

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from satori_b200 import build
    build.build()
    from satori_b200 import _lib
    return _lib


def test_library_exports_every_header_symbol(lib):
    declared = lib.header_symbols(os.path.join(ROOT, "include", "satori_cuda.h"))
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", lib.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    L = lib.lib()
    for s in declared:
        assert getattr(L, s) is not None
    assert set(lib.EXPORTED) == set(declared)


def test_library_reports_its_target(lib):
    assert lib.version().endswith("sm_100a")


def test_init_fails_loudly_without_a_gpu(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from satori_b200 import Context, SatoriError
    with pytest.raises(SatoriError):
        Context(0)


def test_quantized_shape_rules():
    from satori_b200 import ArgumentError, QuantizedMatrixShape
    s = QuantizedMatrixShape(11008, 4096, 1)
    assert (s.block_elements, s.block_bytes, s.byte_length) == (32, 18, 25362432)
    assert QuantizedMatrixShape(4096, 4096, 0).byte_length == 17825792
    for bad in ((0, 32), (1, 33), (1, 0)):
        with pytest.raises(ArgumentError):
            QuantizedMatrixShape(bad[0], bad[1], 0)


def test_ternary2_geometry_matches_benchmark_byte_counts():
    """Ternary2Shape.ByteLength (Ternary2Shape.cs:14) at the benchmark shapes."""
    from satori_b200 import ternary2_byte_length
    assert ternary2_byte_length(4096, 4096, 64) == 5242880
    assert ternary2_byte_length(4096, 4096, 128) == 4718592
    assert ternary2_byte_length(4096, 4096, 256) == 4456448
    assert ternary2_byte_length(1024, 1024, 128) == 294912
    assert ternary2_byte_length(2048, 2048, 128) == 1179648


def test_stq2_header_codec_kat():
    """MappedTernary2Tests.cs:40-46: the exact 32-byte header of a 1x1 block-64 matrix."""
    from satori_b200 import InvalidDataError, stq2_header, stq2_read_header
    kat = golden()["stq2_header_kat"]["expected_hex"]
    assert stq2_header(1, 1, 64).hex() == kat
    assert stq2_read_header(bytes.fromhex(kat)) == (1, 1, 64)
    for index in (0, 4, 6, 8, 16, 20, 24):
        h = bytearray(bytes.fromhex(kat))
        h[index] ^= 0xFF
        with pytest.raises(InvalidDataError):
            stq2_read_header(bytes(h))


def test_no_product_module_imports_the_oracle():
    """The product path never routes through the CPU oracle."""
    pkg = os.path.join(ROOT, "satori_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in text, f
