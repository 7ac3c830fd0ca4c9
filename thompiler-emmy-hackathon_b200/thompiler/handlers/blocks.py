"""Statements that contain a body: Tile, Loop, StridedLoop, Cond.

Tile maps one cell of the iteration space to one thread: the thread's
global id ``ctaid.x * ntid.x + tid.x`` is bounds-checked against the cell
count (the launch may carry more threads than cells, e.g. p00: 64 cells on
256 threads) and decoded row-major into the axis variables.  The semantics
are those of the reference's thompiler/handlers/blocks.py:25-76; the id is
kept in 64 bits when the space has 2^31 cells or more instead of failing.

Loops are emitted in rotated form (one test before entry, one conditional
branch per iteration at the bottom).  A loop whose variable indexes a
register fragment is unrolled at compile time, since registers cannot be
indexed at run time; so is a loop the IR marks ``unroll`` when its bounds
are static and its trip count small.
"""

from __future__ import annotations

from math import prod
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.handlers.mma import indexes_fragment
from thompiler.lowering import expr
from thompiler.lowering.types import dtype_of

if TYPE_CHECKING:
    from thompiler.walk import Walker

MAX_UNROLL = 16


def emit_tile(w: "Walker", tile: ir.Tile) -> None:
    em = w.em
    if tile.aux_threads:
        raise NotImplementedError(f"no lowering for a tile that adds {tile.aux_threads} helper threads")
    extents = tile.extents
    n = tile.n_elements
    em.note(tile.pretty())
    ctaid, ntid, tid = em.tmps("b32", 3)
    em.ins(f"mov.u32 {ctaid}, %ctaid.x")
    em.ins(f"mov.u32 {ntid}, %ntid.x")
    em.ins(f"mov.u32 {tid}, %tid.x")
    end = em.label("tile_end")
    past = em.tmp("pred")
    if n < 2 ** 31:
        gid = em.value("_gid", "b32")
        em.ins(f"mad.lo.u32 {gid}, {ctaid}, {ntid}, {tid}")
        em.ins(f"setp.ge.u32 {past}, {gid}, {n}")
        em.ins(f"@{past} bra {end}")
        for i, axis in enumerate(tile.axes):
            stride = prod(extents[i + 1:])
            reg = em.value(axis.name, "b32")
            if i == 0:
                em.ins(f"mov.u32 {reg}, {gid}" if stride == 1 else f"div.u32 {reg}, {gid}, {stride}")
            elif stride == 1:
                em.ins(f"rem.u32 {reg}, {gid}, {extents[i]}")
            else:
                q = em.tmp("b32")
                em.ins(f"div.u32 {q}, {gid}, {stride}")
                em.ins(f"rem.u32 {reg}, {q}, {extents[i]}")
    else:
        if max(extents) >= 2 ** 31:
            raise NotImplementedError(f"Tile axis with 2^31 or more cells: {extents}")
        gid = em.tmp("b64")
        t = em.tmp("b64")
        em.ins(f"mul.wide.u32 {gid}, {ctaid}, {ntid}")
        em.ins(f"cvt.u64.u32 {t}, {tid}")
        em.ins(f"add.u64 {gid}, {gid}, {t}")
        em.ins(f"setp.ge.u64 {past}, {gid}, {n}")
        em.ins(f"@{past} bra {end}")
        for i, axis in enumerate(tile.axes):
            stride = prod(extents[i + 1:])
            q = em.tmp("b64")
            em.ins(f"div.u64 {q}, {gid}, {stride}")
            if i:
                em.ins(f"rem.u64 {q}, {q}, {extents[i]}")
            em.ins(f"cvt.u32.u64 {em.value(axis.name, 'b32')}, {q}")
    w.body(tile.body)
    em.place(end)


def seed_accumulators(w: "Walker", body: tuple) -> None:
    """Set each accumulator folded directly in ``body`` to its op's identity."""
    em = w.em
    seen: set[str] = set()
    for s in body:
        if not isinstance(s, ir.Accum) or s.name in seen:
            continue
        seen.add(s.name)
        ty = dtype_of(s.dtype, f"Accum {s.name}")
        ident = s.op.identity
        if ident is None:
            raise ValueError(f"Accum {s.name}: {s.op.name} has no identity")
        reg = em.value(s.name, ty.reg)
        em.ins(f"mov.{ty.mov} {reg}, {ty.imm(ident)}")


def static_extent(axis: ir.Axis) -> str:
    if not axis.extent.is_static:
        raise NotImplementedError(f"loop over {axis.name} with a non-static extent")
    return str(axis.extent.as_static())


def emit_loop(w: "Walker", loop: ir.Loop) -> None:
    w.em.note(loop.pretty())
    body = _with_carried_state(w, loop)
    if loop.seed:
        seed_accumulators(w, loop.body)
    counted_loop(w, loop.axis.name, "0", static_extent(loop.axis), "1", body, loop.unroll)


def _with_carried_state(w: "Walker", loop) -> tuple:
    """The loop's body, bracketed per step when it sets carried state (handlers/carry.py)."""
    from thompiler.handlers.carry import carries_in, open_cells
    if not carries_in(loop.body) and not getattr(loop, "carries", ()):
        return loop.body
    begin, end = open_cells(w, loop)
    return (begin, *loop.body, end)


def emit_strided_loop(w: "Walker", loop: ir.StridedLoop) -> None:
    w.em.note(loop.pretty())
    if loop.seed:
        seed_accumulators(w, loop.body)
    body = _with_carried_state(w, loop)
    start = expr.int_operand(w, loop.start)
    bound = expr.int_operand(w, loop.end) if loop.end is not None else static_extent(loop.axis)
    step = expr.int_operand(w, loop.step) if isinstance(loop.step, ir.Expr) else str(int(loop.step))
    counted_loop(w, loop.axis.name, start, bound, step, body, loop.unroll)


def counted_loop(w: "Walker", var: str, start: str, bound: str, step: str, body: tuple,
                 unroll: object = False) -> None:
    consts = all(expr.is_imm(x) for x in (start, bound, step))
    if indexes_fragment(var, body):
        if not consts:
            raise NotImplementedError(f"loop over {var} indexes a fragment but its bounds are not constants")
        unrolled_loop(w, var, int(start), int(bound), int(step), body)
        return
    if consts and unroll and int(step) > 0:
        trips = max(0, -(-(int(bound) - int(start)) // int(step)))
        if trips <= MAX_UNROLL:
            unrolled_loop(w, var, int(start), int(bound), int(step), body)
            return
    rolled_loop(w, var, start, bound, step, body)


def rolled_loop(w: "Walker", var: str, start: str, bound: str, step: str, body: tuple) -> None:
    """for (var = start; var < bound; var += step) -- signed, like C ``int``."""
    em = w.em
    reg = em.value(var, "b32")
    top, done = em.label("loop"), em.label("loop_end")
    em.ins(f"mov.s32 {reg}, {start}")
    if not (expr.is_imm(start) and expr.is_imm(bound) and int(start) < int(bound)):
        skip = em.tmp("pred")
        em.ins(f"setp.ge.s32 {skip}, {reg}, {bound}")
        em.ins(f"@{skip} bra {done}")
    em.place(top)
    w.body(body)
    again = em.tmp("pred")
    em.ins(f"add.s32 {reg}, {reg}, {step}")
    em.ins(f"setp.lt.s32 {again}, {reg}, {bound}")
    em.ins(f"@{again} bra {top}")
    em.place(done)


def unrolled_loop(w: "Walker", var: str, start: int, bound: int, step: int, body: tuple) -> None:
    if step <= 0:
        raise ValueError(f"loop over {var} with step {step}")
    outer = w.consts.get(var)
    for v in range(start, bound, step):
        w.em.note(f"unrolled: {var} = {v}")
        w.consts[var] = v
        w.body(body)
    if outer is None:
        w.consts.pop(var, None)
    else:
        w.consts[var] = outer


def emit_cond(w: "Walker", cond: ir.Cond) -> None:
    em = w.em
    em.note(cond.pretty())
    p = expr.pred_operand(w, cond.cond)
    end = em.label("if_end")
    if cond.else_body:
        other = em.label("else")
        em.ins(f"@!{p} bra {other}")
        w.body(cond.body)
        em.ins(f"bra {end}")
        em.place(other)
        w.body(cond.else_body)
    else:
        em.ins(f"@!{p} bra {end}")
        w.body(cond.body)
    em.place(end)
