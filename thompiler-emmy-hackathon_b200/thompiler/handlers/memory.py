"""Shared memory and barriers: Smem, Sync.

Smem arrays are laid out by the launch contract, as emmy's renderer and the
reference do (thompiler/handlers/memory.py:35-83 of the reference): when
meta.json's ``smem_bytes`` is 0 each array is its own static ``.shared``
symbol (at most 48 KiB in total); otherwise every array is a region of one
dynamic ``.extern .shared`` pool of ``smem_bytes``, placed in declaration
order at its alignment.  The pool symbol is declared 1024-byte aligned so
swizzled slabs (align=1024 in the IR) keep their alignment.

Sync: ``bar.sync 0`` (CTA), ``bar.warp.sync`` (warp), or a named barrier
``bar.sync id, count``.
"""

from __future__ import annotations

from math import prod
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.lowering.address import SharedArray
from thompiler.lowering.types import SMEM_TYPES

if TYPE_CHECKING:
    from thompiler.walk import Walker

STATIC_LIMIT = 48 * 1024
POOL = "smem_pool"
POOL_ALIGN = 1024


def _round_up(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def emit_smem(w: "Walker", s: ir.Smem) -> None:
    if s.dtype not in SMEM_TYPES:
        raise NotImplementedError(f"Smem {s.name} of type {s.dtype!r}")
    ty = SMEM_TYPES[s.dtype]
    extents = tuple(int(e) for e in s.extents)
    known = w.smem.get(s.name)
    if known is not None:
        if known.extents != extents or known.ty != ty:
            raise ValueError(f"Smem {s.name} declared twice with different shapes")
        return
    nbytes = prod(extents) * ty.nbytes
    align = max(int(s.align or 0), ty.nbytes)
    pool = w.kernel.dynamic_smem_bytes
    if pool == 0:
        total = sum(a.nbytes for a in w.smem.values()) + nbytes
        if total > STATIC_LIMIT:
            raise ValueError(f"{total} bytes of static shared memory, above {STATIC_LIMIT}, "
                             "but meta.json's smem_bytes is 0")
        arr = SharedArray(s.name, f"s_{s.name}", 0, extents, ty, nbytes)
        w.em.module(f".shared .align {align} .b8 {arr.symbol}[{nbytes}]")
    else:
        if align > POOL_ALIGN:
            raise NotImplementedError(f"Smem {s.name} needs align {align} > {POOL_ALIGN}")
        w.em.module(f".extern .shared .align {POOL_ALIGN} .b8 {POOL}[]")
        start = _round_up(max((a.offset + a.nbytes for a in w.smem.values()), default=0), align)
        if start + nbytes > pool:
            raise ValueError(f"Smem {s.name} ends at byte {start + nbytes}, past the {pool}-byte "
                             "pool of meta.json's smem_bytes")
        arr = SharedArray(s.name, POOL, start, extents, ty, nbytes)
    w.smem[s.name] = arr
    w.em.note(s.pretty() + (f" (pool + {arr.offset})" if pool else ""))


def emit_sync(w: "Walker", s: ir.Sync) -> None:
    em = w.em
    em.note(s.pretty())
    if s.warp:
        if s.barrier_id:
            raise ValueError("a warp Sync cannot carry a named barrier id")
        em.ins("bar.warp.sync -1")
    elif not s.barrier_id:
        em.ins("bar.sync 0")
    else:
        if s.count is None or not 1 <= int(s.barrier_id) <= 15:
            raise ValueError(f"named Sync needs an id in 1..15 and a count, got "
                             f"id={s.barrier_id} count={s.count}")
        em.ins(f"bar.sync {int(s.barrier_id)}, {int(s.count)}")
