"""Lowering building blocks: C integer folding, swizzle, immediates."""

import struct

from thompiler.lowering.address import swizzle_element, swizzle_params
from thompiler.lowering.expr import fold
from thompiler.lowering.types import F16, F32, F64, I32


def test_fold_truncates_like_c():
    assert fold("/", 7, 2) == 3 and fold("/", -7, 2) == -3 and fold("/", 7, -2) == -3
    assert fold("%", -7, 2) == -1 and fold("%", 7, -2) == 1
    assert fold("*", 6, 7) == 42 and fold("-", 1, 5) == -4


def test_swizzle_modes():
    assert swizzle_params("B128") == (6, 7) and swizzle_params("B64") == (6, 3)
    assert swizzle_params("B32") == (6, 1) and swizzle_params("B128@7") == (7, 7)
    assert swizzle_params("NONE") is None
    # row r (64 halves) of a B128 slab: chunk c lands in chunk c ^ (r & 7)
    for r in range(16):
        for c in range(8):
            e = r * 64 + c * 8
            assert swizzle_element(e, "B128") == r * 64 + ((c ^ (r & 7)) * 8)
    # a swizzle is a permutation of each 1024-element slab
    assert sorted(swizzle_element(e, "B128") for e in range(1024)) == list(range(1024))


def test_immediates():
    assert F32.imm(1.0) == "0f3F800000"
    assert F32.imm(-1e30) == "0f%08X" % struct.unpack("<I", struct.pack("<f", -1e30))[0]
    assert F64.imm(1.0) == "0d3FF0000000000000"
    assert F16.imm(1.0) == "0x3C00"
    assert I32.imm(7) == "7"


def test_wide_buffer_index_expressions_are_64_bit(tmp_path):
    """A buffer of 2^31 or more elements: the whole index expression (a0 * 4 + u) is evaluated
    in 64-bit arithmetic, not widened after a 32-bit product that would wrap past 2^31."""
    from thompiler import compiler, load, synth
    n = (1 << 31) + (1 << 20)
    d = synth.pointwise_package(tmp_path / "pw", n, "relu_mul")
    ptx = compiler.compile_kernel(load.load(str(d / "k_mul_pointwise.ir.json")))
    assert "mul.lo.s64" in ptx
    assert "mul.lo.s32" not in ptx                       # no 32-bit index product anywhere
    small = synth.pointwise_package(tmp_path / "pw_small", 1 << 20, "relu_mul")
    ptx_small = compiler.compile_kernel(load.load(str(small / "k_mul_pointwise.ir.json")))
    assert "mul.lo.s64" not in ptx_small                 # small buffers keep the 32-bit form
