"""buffer[index] -> an address operand.

Two memories:
  * a kernel parameter lives in global memory: its base register
    (``%g_<buffer>``) plus the element's byte offset.  The offset is formed
    with one ``mad.wide.s32`` from a 32-bit flat index when the buffer has
    fewer than 2^31 elements, and in 64-bit arithmetic above that, so a
    buffer of any size is addressed correctly (the reference's 32-bit flat
    index, thompiler/lowering/address.py:42-79, stops at 2^31 elements);
  * an Smem array lives in shared memory: a 32-bit offset from the array's
    symbol, optionally permuted by a swizzle.

Every function returns an operand that goes inside ``[...]``: a register,
or ``register+imm`` / ``symbol+imm`` when the offset is a compile-time
constant (so no instruction is spent on it).

Swizzles follow emmy's element-index convention (``LDMATRIX_SWIZZLE_XOR``,
mirrored by the reference's address.py:115-150): for mode ``(shift, mask)``
the element ``e`` of a slab is stored at ``e ^ (((e >> shift) & mask) << 3)``,
i.e. 8-element chunks of a row are XOR-ed with the row's low bits.  Modes
B128 = (6, 7), B64 = (6, 3), B32 = (6, 1); ``<mode>@<s>`` overrides the shift.
Writers and readers of one slab must use the same mode, so this table is a
data-format convention, not a choice of this backend.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING

from thompiler.lowering.expr import int_operand, int_operand_wide, is_imm
from thompiler.lowering.types import Ty

if TYPE_CHECKING:
    from thompiler.load import Param
    from thompiler.walk import Walker

WIDE_ELEMENTS = 2 ** 31


@dataclass
class SharedArray:
    name: str
    symbol: str           # PTX symbol the array is addressed from
    offset: int           # byte offset of the array from the symbol
    extents: tuple[int, ...]
    ty: Ty
    nbytes: int


SWIZZLES: dict[str, tuple[int, int]] = {"B128": (6, 0x7), "B64": (6, 0x3), "B32": (6, 0x1)}


def swizzle_params(mode: str) -> tuple[int, int] | None:
    if mode in ("NONE", None, ""):
        return None
    base, sep, shift = mode.partition("@")
    if base not in SWIZZLES:
        raise NotImplementedError(f"no shared-memory layout {mode!r}")
    dshift, mask = SWIZZLES[base]
    return (int(shift) if sep else dshift, mask)


def swizzle_element(e: int, mode: str) -> int:
    p = swizzle_params(mode)
    if p is None:
        return e
    shift, mask = p
    return e ^ (((e >> shift) & mask) << 3)


def flat_index(w: "Walker", shape: tuple[int, ...], index: tuple, what: str) -> str:
    """Row-major element offset of ``index`` in ``shape`` (32-bit)."""
    if len(index) != len(shape):
        raise ValueError(f"{what}: {len(index)} indices for shape {shape}")
    if not index:
        return "0"
    em = w.em
    flat = int_operand(w, index[0])
    for size, e in zip(shape[1:], index[1:]):
        i = int_operand(w, e)
        if is_imm(flat) and is_imm(i):
            flat = str(int(flat) * size + int(i))
        elif is_imm(flat) and int(flat) == 0:
            flat = i
        else:
            out = em.tmp("b32")
            em.ins(f"mad.lo.s32 {out}, {flat}, {size}, {i}")
            flat = out
    return flat


def _flat_index_wide(w: "Walker", shape: tuple[int, ...], index: tuple) -> str:
    """Row-major element offset in 64-bit arithmetic (b64 register or imm)."""
    em = w.em
    flat = None
    for k, (size, e) in enumerate(zip(shape, index)):
        iw = int_operand_wide(w, e)
        if flat is None:
            flat = iw
        elif is_imm(flat) and is_imm(iw):
            flat = str(int(flat) * size + int(iw))
        else:
            out = em.tmp("b64")
            em.ins(f"mad.lo.s64 {out}, {flat}, {size}, {iw}")
            flat = out
    return flat or "0"


def global_address(w: "Walker", p: "Param", index: tuple) -> str:
    em = w.em
    base = em.buffer_reg(p.name)
    if not index:
        if p.shape and p.nelems != 1:
            raise ValueError(f"{p.name}: no index for shape {p.shape}")
        return base
    if p.nelems >= WIDE_ELEMENTS:
        flat = _flat_index_wide(w, p.shape, index)
        if is_imm(flat):
            off = int(flat) * p.ty.nbytes
            return base if off == 0 else f"{base}+{off}"
        out = em.tmp("b64")
        em.ins(f"mad.lo.s64 {out}, {flat}, {p.ty.nbytes}, {base}")
        return out
    flat = flat_index(w, p.shape, index, p.name)
    if is_imm(flat):
        off = int(flat) * p.ty.nbytes
        return base if off == 0 else f"{base}+{off}"
    out = em.tmp("b64")
    em.ins(f"mad.wide.s32 {out}, {flat}, {p.ty.nbytes}, {base}")
    return out


def shared_element_address(w: "Walker", arr: SharedArray, flat: str, swizzle: str = "NONE") -> str:
    """Address of flat element ``flat`` of a shared array, after ``swizzle``."""
    em = w.em
    p = swizzle_params(swizzle)
    if p is not None:
        if is_imm(flat):
            flat = str(swizzle_element(int(flat), swizzle))
        else:
            shift, mask = p
            t1, t2 = em.tmp("b32"), em.tmp("b32")
            em.ins(f"shr.u32 {t1}, {flat}, {shift}")
            em.ins(f"and.b32 {t1}, {t1}, {mask}")
            em.ins(f"shl.b32 {t1}, {t1}, 3")
            em.ins(f"xor.b32 {t2}, {flat}, {t1}")
            flat = t2
    if is_imm(flat):
        off = arr.offset + int(flat) * arr.ty.nbytes
        return arr.symbol if off == 0 else f"{arr.symbol}+{off}"
    base = em.tmp("b32")
    em.ins(f"mov.u32 {base}, {arr.symbol}")
    out = em.tmp("b32")
    em.ins(f"mad.lo.s32 {out}, {flat}, {arr.ty.nbytes}, {base}")
    if arr.offset:
        return f"{out}+{arr.offset}"
    return out


def shared_address(w: "Walker", arr: SharedArray, index: tuple, swizzle: str = "NONE") -> str:
    return shared_element_address(w, arr, flat_index(w, arr.extents, index, arr.name), swizzle)


def access(w: "Walker", buffer: str, index: tuple, swizzle: str = "NONE") -> tuple[str, str, Ty, bool]:
    """(state space, address operand, element type, read-only global?)."""
    p = w.kernel.param(buffer)
    if p is not None:
        if swizzle not in ("NONE", None, ""):
            raise ValueError(f"{buffer} lives in global memory; swizzle {swizzle} applies to shared arrays only")
        return "global", global_address(w, p, index), p.ty, not p.written
    arr = w.smem.get(buffer)
    if arr is not None:
        return "shared", shared_address(w, arr, index, swizzle), arr.ty, False
    raise ValueError(f"{buffer!r}: no kernel parameter or Smem array has this name")
