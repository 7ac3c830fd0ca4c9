"""Asynchronous global -> shared copies: CpAsyncCopy / Commit / Wait.

In the generic lowering each CpAsyncCopy stays one per-thread ``cp.async``
of 4, 8 or 16 bytes (``.cg`` bypasses L1 and takes only 16 bytes; ``.ca``
for the smaller sizes), its destination being the Smem element at
``smem_index`` plus the thread's own (row, col) ``lane_index`` in the copy
stripe, after the slab's swizzle -- the IR reference's definition, as the
reference implements it in thompiler/handlers/cp_async.py:20-47.  The
tuned matmul family replaces these copies by TMA bulk tensor copies.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.lowering import address, expr

if TYPE_CHECKING:
    from thompiler.walk import Walker

CACHE = {4: "ca", 8: "ca", 16: "cg"}


def emit_cp_async_copy(w: "Walker", c: ir.CpAsyncCopy) -> None:
    em = w.em
    em.note(c.pretty())
    if c.nbytes not in CACHE:
        raise ValueError(f"cp.async of {c.nbytes} bytes (4, 8 or 16 only)")
    arr = w.smem.get(c.smem)
    src = w.kernel.param(c.src)
    if arr is None or src is None:
        raise ValueError(f"cp.async from {c.src!r} to {c.smem!r} needs a kernel parameter "
                         "source and an Smem destination")
    elem = address.flat_index(w, arr.extents, tuple(c.smem_index), arr.name)
    if c.lane_index is not None:
        row, col = c.lane_index
        lane = ir.BinaryExpr("+", ir.BinaryExpr("*", row, ir.Literal(arr.extents[-1], "int")), col)
        elem = expr.add_ints(w, elem, expr.int_operand(w, lane))
    dst = address.shared_element_address(w, arr, elem, c.swizzle)
    gsrc = address.global_address(w, src, tuple(c.src_index))
    em.ins(f"cp.async.{CACHE[c.nbytes]}.shared.global [{dst}], [{gsrc}], {c.nbytes}")


def emit_cp_async_commit(w: "Walker", c: ir.CpAsyncCommit) -> None:
    w.em.ins("cp.async.commit_group")


def emit_cp_async_wait(w: "Walker", c: ir.CpAsyncWait) -> None:
    w.em.ins(f"cp.async.wait_group {int(c.group)}")
