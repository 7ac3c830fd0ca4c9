"""Element types: how an IR dtype is spelled in PTX.

One ``Ty`` per supported type carries everything an instruction template
needs: the arithmetic suffix (``f32`` / ``s32``), the suffix of plain moves
(``ld`` / ``st`` / ``mov``, where f16 is ``b16``), the register class its
values live in, and its size.  The reference keeps the same information in
thompiler/lowering/types.py:24-84; this table adds the integer widths the
64-bit address path needs and f16 arithmetic, which sm_100a executes natively.

Register classes are the PTX ``.reg`` kinds the emitter declares:
``pred b16 b32 b64 f32 f64``.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass


@dataclass(frozen=True)
class Ty:
    name: str        # IR dtype name: "f32", "f16", "f64", "i32", "i64"
    kind: str        # "float" or "int"
    ptx: str         # arithmetic suffix: f32, f16, f64, s32, s64
    mov: str         # suffix of ld / st / mov / shfl payloads: f32, b16, f64, s32, s64
    reg: str         # register class
    nbytes: int

    @property
    def is_float(self) -> bool:
        return self.kind == "float"

    def imm(self, value: float | int) -> str:
        """``value`` as a PTX immediate of this type.

        Floats are written as their IEEE bits (``0f3F800000``, ``0d3FF0...``)
        so the value is exact and locale-free; rounding to f32 follows
        ``struct`` (round to nearest, like a C float literal)."""
        if not self.is_float:
            return str(int(value))
        if self.ptx == "f32":
            return "0f%08X" % struct.unpack("<I", struct.pack("<f", float(value)))[0]
        if self.ptx == "f64":
            return "0d%016X" % struct.unpack("<Q", struct.pack("<d", float(value)))[0]
        if self.ptx == "f16":
            # PTX has no f16 immediate: a b16 register is loaded with the bits.
            return "0x%04X" % struct.unpack("<H", struct.pack("<e", float(value)))[0]
        raise NotImplementedError(f"{self.name} immediate")


F16 = Ty("f16", "float", "f16", "b16", "b16", 2)
F32 = Ty("f32", "float", "f32", "f32", "f32", 4)
F64 = Ty("f64", "float", "f64", "f64", "f64", 8)
I32 = Ty("i32", "int", "s32", "s32", "b32", 4)
I64 = Ty("i64", "int", "s64", "s64", "b64", 8)
PRED = Ty("pred", "int", "pred", "pred", "pred", 0)
# bytes: the packed fp4 operands and ue8m0 block scales of block-scaled MMAs (loaded into 32-bit
# registers, zero-extended)
U8 = Ty("u8", "int", "u8", "u8", "b32", 1)
# register-fragment element types that no buffer holds: fp4 (e2m1, eight per 32-bit register) and
# the ue8m0 block-scale bytes (four per register)
E2M1 = Ty("e2m1", "float", "e2m1", "b32", "b32", 0)
UE8M0 = Ty("ue8m0", "int", "ue8m0", "b32", "b32", 1)
FRAGMENT_TYPES: dict[str, Ty] = {"e2m1": E2M1, "fp4": E2M1, "ue8m0": UE8M0}

# Buffer / value dtypes by IR name: the float types of the problems, and bytes for the
# block-scaled fp4 statements' packed operands and scales.
BUFFER_TYPES: dict[str, Ty] = {"f16": F16, "f32": F32, "f64": F64, "u8": U8, "uint8": U8}

# Smem.dtype is the C element type emmy renders, not an IR dtype.
SMEM_TYPES: dict[str, Ty] = {"__half": F16, "half": F16, "float": F32, "double": F64,
                             # 8-byte words: the mbarrier arrays of the TMA statements
                             "uint64_t": I64, "int64_t": I64, "unsigned long long": I64, "long long": I64,
                             "u64": I64, "i64": I64,
                             # bytes: packed fp4 tiles and block scales
                             "uint8_t": U8, "unsigned char": U8, "u8": U8}

# Literal.dtype -> type of the literal.
LITERAL_TYPES: dict[str, Ty] = {"int": I32, "float": F32}

# Register class -> the value type a named register of that class holds.
REG_VALUE_TYPE: dict[str, Ty] = {"b16": F16, "f32": F32, "f64": F64, "b32": I32, "b64": I64}


def dtype_of(dtype: object, what: str) -> Ty:
    """The Ty of an IR dtype (a DataType, its name, or None meaning f32)."""
    if dtype is None:
        return F32
    name = str(getattr(dtype, "name", dtype))
    ty = BUFFER_TYPES.get(name)
    if ty is None:
        raise NotImplementedError(f"{what}: dtype {name!r} is not supported")
    return ty
