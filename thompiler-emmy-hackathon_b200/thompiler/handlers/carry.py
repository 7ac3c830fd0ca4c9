"""Carried state: Carry, Pre (and Loop.carries).

The IR reference (TASK.md:104-105 of the reference) defines carried state for loops that pass
values from one step to the next (a scan): ``Carry(name, value, index, seed, dtype)`` sets
the next value of cell ``index`` of carrier ``name``; ``Pre(name, carrier, index)`` reads a
cell -- inside the carrying loop the previous step's value (the seed on the first step), after
the loop the final value.  Reads within a step see the previous state, and cells a step does
not set keep their values.  The reference compiler has no lowering for these.

A Carry belongs to its innermost enclosing loop (``Loop.carries``, when the IR lists it, must
name only carriers the body sets).  Every cell (carrier, constant index) of that loop is two
registers: ``cur`` is seeded before the loop, copied to ``next`` when a step starts and
replaced by ``next`` when it ends; ``Carry`` writes ``next``, ``Pre`` reads ``cur``.  A cell
index must be a compile-time constant (literals and unrolled loop variables).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Any

from thompiler import ir
from thompiler.lowering import expr
from thompiler.lowering.types import F32, I32, REG_VALUE_TYPE, dtype_of

if TYPE_CHECKING:
    from thompiler.walk import Walker


@dataclass(frozen=True)
class StepBegin(ir.Stmt):
    """Internal: the start of one step of a carrying loop (next := cur for its cells)."""
    cells: tuple = ()


@dataclass(frozen=True)
class StepEnd(ir.Stmt):
    """Internal: the end of one step of a carrying loop (cur := next for its cells)."""
    cells: tuple = ()


def _const(w: "Walker", e: Any) -> int:
    if isinstance(e, bool):
        raise NotImplementedError("a boolean carried-state cell index")
    if isinstance(e, int):
        return e
    if isinstance(e, ir.Literal) and isinstance(e.value, int):
        return int(e.value)
    if isinstance(e, ir.Var) and e.name in w.consts:
        return w.consts[e.name]
    if isinstance(e, ir.BinaryExpr) and e.op in ("+", "-", "*", "/", "%"):
        return expr.fold(e.op, _const(w, e.left), _const(w, e.right))
    raise NotImplementedError(f"carried-state cell {ir.pretty(e)}: only indices that fold to a constant are lowered")


def cell_key(w: "Walker", carrier: str, index) -> tuple:
    idx = index if isinstance(index, tuple) else (index,)
    return (carrier, tuple(_const(w, i) for i in idx))


def carries_in(stmts) -> list:
    """The Carry statements a loop with body ``stmts`` owns: those not inside a nested loop (a
    Carry belongs to its innermost enclosing loop)."""
    out = []
    for s in stmts:
        if isinstance(s, ir.Carry):
            out.append(s)
        elif isinstance(s, ir.Cond):
            out += carries_in(s.body) + carries_in(s.else_body)
    return out


def _operand(w: "Walker", v, ty) -> str:
    em = w.em
    if isinstance(v, str):
        return em.get(v)
    if isinstance(v, ir.Var) and v.name not in w.consts:
        return em.get(v.name)
    if isinstance(v, ir.Literal):
        return ty.imm(float(v.value) if ty.is_float else int(v.value))
    if ty is I32:
        return expr.int_operand(w, v)
    raise NotImplementedError(f"carried value {ir.pretty(v)}")


def open_cells(w: "Walker", loop) -> tuple:
    """Declare and seed the cells of a carrying loop; the (begin, end) markers for its body."""
    carriers = set(getattr(loop, "carries", ()) or ())
    cells = {}
    for c in carries_in(loop.body):
        key = cell_key(w, c.name, c.index)
        if key in cells:
            continue
        ty = dtype_of(c.dtype, f"Carry {c.name}") if c.dtype is not None else F32
        cells[key] = (c, ty)
    missing = carriers - {k[0] for k in cells}
    if missing:
        raise ValueError(f"loop over {loop.axis.name} carries {sorted(missing)} but never sets them")
    em = w.em
    w.carry_cells = getattr(w, "carry_cells", {})
    keys = []
    for key, (c, ty) in cells.items():
        tag = "_".join(str(i) for i in key[1]) or "s"
        cur = em.value(f"{key[0]}__cell_{tag}", ty.reg)
        nxt = em.tmp(ty.reg)
        seed = c.seed if c.seed is not None else ir.Literal(0.0 if ty.is_float else 0, "float" if ty.is_float else "int")
        em.ins(f"mov.{ty.mov} {cur}, {_operand(w, seed, ty)}")
        w.carry_cells[key] = (cur, nxt, ty)
        keys.append(key)
    return StepBegin(tuple(keys)), StepEnd(tuple(keys))


def emit_step_begin(w: "Walker", s: StepBegin) -> None:
    for key in s.cells:
        cur, nxt, ty = w.carry_cells[key]
        w.em.ins(f"mov.{ty.mov} {nxt}, {cur}")


def emit_step_end(w: "Walker", s: StepEnd) -> None:
    for key in s.cells:
        cur, nxt, ty = w.carry_cells[key]
        w.em.ins(f"mov.{ty.mov} {cur}, {nxt}")


def emit_carry(w: "Walker", c: ir.Carry) -> None:
    em = w.em
    em.note(c.pretty())
    key = cell_key(w, c.name, c.index)
    cell = getattr(w, "carry_cells", {}).get(key)
    if cell is None:
        raise ValueError(f"Carry {c.name}{list(key[1])} outside a loop that carries {c.name}")
    cur, nxt, ty = cell
    v = _operand(w, c.value, ty)
    if isinstance(c.value, str) and REG_VALUE_TYPE[em.cls_of(c.value)] is not ty:
        raise TypeError(f"Carry {c.name}: a {REG_VALUE_TYPE[em.cls_of(c.value)].name} value into a {ty.name} cell")
    em.ins(f"mov.{ty.mov} {nxt}, {v}")


def emit_pre(w: "Walker", p: ir.Pre) -> None:
    em = w.em
    em.note(p.pretty())
    key = cell_key(w, p.carrier, p.index)
    cell = getattr(w, "carry_cells", {}).get(key)
    if cell is None:
        raise ValueError(f"Pre {p.name}: carrier {p.carrier}{list(key[1])} is not carried by an enclosing or "
                         "earlier loop")
    cur, _, ty = cell
    em.ins(f"mov.{ty.mov} {em.value(p.name, ty.reg)}, {cur}")
