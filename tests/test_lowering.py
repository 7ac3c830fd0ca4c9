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
